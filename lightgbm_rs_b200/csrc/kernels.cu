// Hand-written sm_100a kernels of the leaf-wise histogram tree learner.
//
// Per split s the host enqueues (no host synchronisation anywhere in a tree):
//   k_prepare(s)   1 CTA  apply split s-1 (Tree::split + child LeafSplits seeding),
//                         BeforeFindBestSplit gates, smaller/larger choice, pool slots
//   k_build        grid   shared-memory-privatised histogram of the smaller child
//   k_fixscan      F CTAs decode + FixHistogram + compaction + parent-smaller
//                         subtraction + REVERSE/FORWARD threshold scans; the last CTA
//                         does the per-leaf and cross-leaf argmax
//   k_partition    grid   stable single-pass partition of the chosen leaf's rows
// All decisions live in GrowCtrl on the device; kernels after a finished tree
// return at once.
#include <cstdio>

#include "kernels.cuh"

namespace lgbm_b200 {

namespace {

constexpr int kBuildThreads = 512;
constexpr int kMinRowsPerBlock = 1024;
constexpr int kScanThreads = 1024;
// The control step sums at most two halves of per-tile partials, one load per tile each.
constexpr int kHalfTiles = kMaxPrivateTiles / 2;
static_assert(kScanThreads == 1024, "the partial-sum halves are the CTA's two 512-thread halves");
constexpr int kPartThreads = 256;
constexpr int kPartItems = 8;
constexpr int kPartTile = kPartThreads * kPartItems;
static_assert(kPartTile == kPartitionTileRows, "partition tile size is part of the host contract");
constexpr long long kSpinLimit = 1ll << 22;


__device__ __forceinline__ bool leaf_buildable(const DevLeafSplits& l) {
  return l.sum_h > 0.0 && l.num_data > 0;  // learner.rs:2477-2481
}

// What a histogram build accumulates into d.raw. Phase 0: the root (all rows of this
// device, identity order, every feature). Phase 1: one child of the split just
// partitioned -- its left rows [begin, begin + left) or right rows [begin + left,
// begin + count) in the partition's destination buffer, features the parent could
// split only. Phase 2: nothing (last split of the tree); the partition's left count
// is still published.
struct BuildTarget {
  int32_t begin, count, buf, mask_leaf;
  bool ok;
};

__device__ __forceinline__ BuildTarget build_target(const GrowDev& d, int phase) {
  const GrowCtrl* c = d.ctrl;
  BuildTarget t{0, 0, 2, -1, false};
  if (c->done) return t;
  if (phase == 0) {
    t.count = (int32_t)d.N;
    t.ok = t.count > 0;
    return t;
  }
  if (phase != 1 || !c->pending) return t;
  const int32_t leaf = c->split_leaf;
  const int32_t beg = d.leaf_begin[leaf];
  const int32_t cnt = d.leaf_count[leaf];
  const int32_t lc = c->part_left_total;
  t.buf = d.leaf_buf[leaf] == 1 ? 0 : 1;
  if (c->build_left) {
    t.begin = beg;
    t.count = lc;
  } else {
    t.begin = beg + lc;
    t.count = cnt - lc;
  }
  t.mask_leaf = leaf;
  t.ok = t.count > 0;
  return t;
}

// Build bookkeeping, once per build launch (block (0,0), thread 0): the non-fused
// partition publishes its left count here for the next split's control step.
__device__ __forceinline__ void build_account(const GrowDev& d, int phase, const BuildTarget& t) {
  if (blockIdx.x != 0 || blockIdx.y != 0 || threadIdx.x != 0) return;
  GrowCtrl* c = d.ctrl;
  if (phase != 0 && !d.fused && !c->done && c->pending)
    d.raw[d.raw_len] = (long long)c->part_left_total;
  if (t.ok) {
    c->num_builds += 1;
    c->rows_built += t.count;
  }
}

// ------------------------------------------------------------------------------------
// Exchange of the accumulated child over peer memory (GrowDev::xranks > 1).
// ------------------------------------------------------------------------------------

__device__ __forceinline__ long long ld_relaxed_sys(const long long* p) {
  long long v;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Entry/exit stamps of a launch into GrowDev's span arrays (thread 0 of every CTA);
// nothing when the spans are off.
struct SpanStamp {
  const GrowDev& d;
  __device__ __forceinline__ explicit SpanStamp(const GrowDev& g) : d(g) {
    if (d.span_start && threadIdx.x == 0) atomicMin(d.span_start + d.span_slot, global_ns());
  }
  __device__ __forceinline__ ~SpanStamp() {
    if (d.span_end && threadIdx.x == 0) atomicMax(d.span_end + d.span_slot, global_ns());
  }
};

// Phase mark p of control step s (thread 0 of the calling CTA; nothing when off).
__device__ __forceinline__ void ctl_mark(const GrowDev& d, int s, int p) {
  if (d.ctl_phase && threadIdx.x == 0) atomicMax(d.ctl_phase + (size_t)s * kStepMarks + p, global_ns());
}

// Phase mark p of a partition launch (thread 0; nothing when off). The launch's split step
// is that of its span slot; `t` is the time to record.
__device__ __forceinline__ void part_mark(const GrowDev& d, bool lookahead, int p,
                                          unsigned long long t) {
  if (d.ctl_phase && threadIdx.x == 0 && d.span_slot >= 1)
    atomicMax(d.ctl_phase + (size_t)((d.span_slot - 1) >> 2) * kStepMarks + kCtlPhases +
                  (lookahead ? 0 : kPartPhases) + p,
              t);
}

// Sum over the ranks of word `off` of each rank's buffer (integers: exact in any order).
// The ranks' buffer pointers are read first and every rank's load is issued before any
// is added, so one round trip over the peer links covers all ranks.
__device__ __forceinline__ long long peer_sum(long long* const* bufs, int ranks, size_t off) {
  const long long* p[kMaxXRanks];
#pragma unroll
  for (int r = 0; r < kMaxXRanks; ++r) p[r] = r < ranks ? bufs[r] : nullptr;
  long long v[kMaxXRanks];
#pragma unroll
  for (int r = 0; r < kMaxXRanks; ++r) v[r] = r < ranks ? ld_relaxed_sys(p[r] + off) : 0ll;
  long long s = 0;
#pragma unroll
  for (int r = 0; r < kMaxXRanks; ++r) s += v[r];
  return s;
}

// Cell `idx` of the accumulated child: the sum over the ranks' buffers of parity xpar
// (integers: exact in any order); on one device, the launch's accumulator.
template <bool PEER>
__device__ __forceinline__ long long raw_sum(const GrowDev& d, size_t idx) {
  if (!PEER) return __ldcg(d.raw + idx);
  const size_t off = (size_t)d.xpar * ((size_t)d.raw_len + 2) + idx;
  return peer_sum(d.xbuf, d.xranks, off);
}

// Waits (thread 0 of a consumer CTA) until every rank has published this rank's current
// exchange count; false after wait_ns without it, or at once when a wait has already run
// out (the caller records kErrSpinTimeout). Each poll reads every rank's flag in one round
// trip (relaxed loads issued together); once all have reached `seq`, one system-scope
// acquire fence orders the caller's later reads of the ranks' buffers after the ranks'
// release stores of those flags.
__device__ __noinline__ bool x_wait_target(const uint32_t* error, int xranks,
                                           const unsigned long long* xflags,
                                           unsigned long long seq, long long wait_ns) {
  if (*reinterpret_cast<const volatile uint32_t*>(error) & kErrSpinTimeout) return false;
  const unsigned long long t0 = global_ns();
  while (true) {
    unsigned long long v[kMaxXRanks];
#pragma unroll
    for (int r = 0; r < kMaxXRanks; ++r)
      v[r] = r < xranks ? (unsigned long long)ld_relaxed_sys(
                              reinterpret_cast<const long long*>(xflags + r))
                        : seq;
    bool ready = true;
#pragma unroll
    for (int r = 0; r < kMaxXRanks; ++r) ready = ready && v[r] >= seq;
    if (ready) break;
    if (global_ns() - t0 > (unsigned long long)wait_ns) return false;
    __nanosleep(64);
  }
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  return true;
}

// The control step's two waits in one polling loop: every rank's accumulator flag at
// `seq`, and, when the pending split was partitioned by a look-ahead, every rank's
// look-ahead flag at `want` (both arrays' loads issued together: one round trip when
// both are ready). One acquire fence after both.
__device__ __noinline__ bool x_wait_both(const uint32_t* error, int xranks,
                                         const unsigned long long* xflags,
                                         unsigned long long seq,
                                         const unsigned long long* laflags,
                                         unsigned long long want, long long wait_ns) {
  if (*reinterpret_cast<const volatile uint32_t*>(error) & kErrSpinTimeout) return false;
  const unsigned long long t0 = global_ns();
  while (true) {
    unsigned long long v[kMaxXRanks], w[kMaxXRanks];
#pragma unroll
    for (int r = 0; r < kMaxXRanks; ++r) {
      v[r] = r < xranks ? (unsigned long long)ld_relaxed_sys(
                              reinterpret_cast<const long long*>(xflags + r))
                        : seq;
      w[r] = (laflags && r < xranks) ? (unsigned long long)ld_relaxed_sys(
                                           reinterpret_cast<const long long*>(laflags + r))
                                     : want;
    }
    bool ready = true;
#pragma unroll
    for (int r = 0; r < kMaxXRanks; ++r) ready = ready && v[r] >= seq && w[r] >= want;
    if (ready) break;
    if (global_ns() - t0 > (unsigned long long)wait_ns) return false;
    __nanosleep(64);
  }
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  return true;
}

// Both waits of the control step: x_wait, then la_wait, as one poll.
template <bool PEER>
__device__ __forceinline__ bool x_la_wait(const GrowDev& d, int s) {
  if (!PEER) return true;
  const GrowCtrl* c = d.ctrl;
  const bool la = d.lookahead && c->pending && c->pend_la;
  return x_wait_both(&c->error, d.xranks, d.xflags,
                     *reinterpret_cast<const volatile unsigned long long*>(d.xseq),
                     la ? d.la_flags : nullptr,
                     la ? c->la_base + (unsigned long long)(s - 1) : 0ull, d.xwait_ns);
}

template <bool PEER>
__device__ __forceinline__ bool x_wait(const GrowDev& d) {
  if (!PEER) return true;
  return x_wait_target(&d.ctrl->error, d.xranks, d.xflags,
                       *reinterpret_cast<const volatile unsigned long long*>(d.xseq),
                       d.xwait_ns);
}

// Cell idx of look-ahead slot `slot`: this device's, or the sum over the ranks.
template <bool PEER>
__device__ __forceinline__ long long la_sum(const GrowDev& d, int slot, size_t idx) {
  const size_t off = (size_t)slot * ((size_t)d.raw_len + 2) + idx;
  if (!PEER) return __ldcg(d.la_raw + off);
  return peer_sum(d.la_xbuf, d.xranks, off);
}

// With several devices, a pending split partitioned by the look-ahead of step s - 2 (the
// (s - 1)-th look-ahead signal of the tree) is read from every rank's slot: wait for all
// ranks' signals. False after the wait limit.
template <bool PEER>
__device__ __forceinline__ bool la_wait(const GrowDev& d, int s) {
  if (!PEER || !d.lookahead) return true;
  const GrowCtrl* c = d.ctrl;
  if (!(c->pending && c->pend_la)) return true;
  const unsigned long long want = c->la_base + (unsigned long long)(s - 1);
  return x_wait_target(&c->error, d.xranks, d.la_flags, want, d.xwait_ns);
}

// After a producer kernel: publish the next exchange count into every rank's flags
// (system-scope release after the producer's completed writes). One warp.
__global__ void k_xsignal(GrowDev d) {
  const int lane = threadIdx.x;
  const unsigned long long seq = *d.xseq + 1;
  __syncwarp();
  __threadfence_system();
  if (lane < d.xranks) {
    unsigned long long* f = d.peer_xflags[lane] + d.xrank;
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(f), "l"(seq) : "memory");
  }
  if (lane == 0) *d.xseq = seq;
}

// After a look-ahead kernel: the same publication for the look-ahead slots.
__global__ void k_lasignal(GrowDev d) {
  const int lane = threadIdx.x;
  const unsigned long long seq = *d.la_seq + 1;
  __syncwarp();
  __threadfence_system();
  if (lane < d.xranks) {
    unsigned long long* f = d.peer_la_flags[lane] + d.xrank;
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(f), "l"(seq) : "memory");
  }
  if (lane == 0) *d.la_seq = seq;
}

// End of a producer launch that publishes its own exchange (self_signal): what k_xsignal
// or k_lasignal would do after the kernel, without a launch of its own. Every thread of
// every CTA calls it after its last write. The CTAs arrive on an acq_rel counter (so the
// last one to arrive has every CTA's writes ordered before it), and the last one resets
// the counter for the next launch of its kind (stream-ordered after this one), fences at
// system scope and releases the next sequence number into every rank's flag.
__device__ __forceinline__ void producer_signal(const GrowDev& d) {
  if (!d.self_signal) return;
  __threadfence();
  __syncthreads();
  if (threadIdx.x != 0) return;
  const int k = d.self_signal - 1;
  uint32_t* cnt = d.arrive + k;
  const uint32_t n = gridDim.x * gridDim.y * gridDim.z;
  uint32_t t;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(t) : "l"(cnt), "r"(1u)
               : "memory");
  if (t != n - 1) return;
  *cnt = 0u;
  unsigned long long* seqp = k == 0 ? d.xseq : d.la_seq;
  unsigned long long* const* flags = k == 0 ? d.peer_xflags : d.peer_la_flags;
  const unsigned long long seq = *seqp + 1;
  __threadfence_system();
  for (int r = 0; r < d.xranks; ++r) {
    unsigned long long* f = flags[r] + d.xrank;
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(f), "l"(seq) : "memory");
  }
  *seqp = seq;
}

// Decoding of the raw integer accumulators into f64 histogram cells. For the
// quantized modes the result equals the reference's f64 fold exactly: every
// dequantized level is an integer multiple of the ulp of the smallest nonzero
// level, so all partial sums of the reference's sequential fold are exact.
__device__ __forceinline__ double decode_g(const DevGhParams& p, long long v) {
  return (double)v * p.unit_g;
}
__device__ __forceinline__ double decode_h(const DevGhParams& p, long long v) {
  if (p.mode == GH_QPACK) {
    const long long hl = v & 0xffffffffll;
    const long long c3 = v >> 32;
    return (double)hl * p.unit_h + (double)c3 * p.v3h;
  }
  return (double)v * p.unit_h;
}

// ------------------------------------------------------------------------------------
// Histogram build: one CTA accumulates a row range of one feature group in shared
// memory with 64-bit integer atomics, then merges into the global raw accumulator.
// ------------------------------------------------------------------------------------

template <int MODE>
struct GhValue;

template <>
struct GhValue<GH_FLOAT> {
  long long a, b;
  __device__ __forceinline__ void load(const void* gh, uint32_t row, const DevGhParams& p,
                                       const long long*, const long long*) {
    const float2 v = reinterpret_cast<const float2*>(gh)[row];
    a = __double2ll_rn((double)v.x * p.scale_g);
    b = __double2ll_rn((double)v.y * p.scale_h);
  }
};

template <>
struct GhValue<GH_QLUT> {
  long long a, b;
  __device__ __forceinline__ void load(const void* gh, uint32_t row, const DevGhParams&,
                                       const long long* lut_g, const long long* lut_h) {
    const uint16_t q = reinterpret_cast<const uint16_t*>(gh)[row];
    a = lut_g[(int)(int8_t)(q & 0xff) + 128];
    b = lut_h[(int)(int8_t)(q >> 8) + 128];
  }
};

// Packed form for num_grad_quant_bins <= 4: qg in [-2,2] (linear levels), qh in [0,4]
// where only level 3 is not a multiple of level 1. One int64 per row:
//   bits 0..20 signed sum of qg | bits 21..41 sum of qh over levels {1,2,4} | bits 42.. count of qh==3
template <>
struct GhValue<GH_QPACK> {
  long long a, b;
  __device__ __forceinline__ void load(const void* gh, uint32_t row, const DevGhParams&,
                                       const long long*, const long long*) {
    const uint16_t q = reinterpret_cast<const uint16_t*>(gh)[row];
    const long long qg = (long long)(int8_t)(q & 0xff);
    const int qh = (int)(int8_t)(q >> 8);
    const long long hl = qh == 3 ? 0 : qh;
    const long long c3 = qh == 3 ? 1 : 0;
    a = qg + (hl << 21) + (c3 << 42);
    b = 0;
  }
};

__device__ __forceinline__ void unpack_qpack(unsigned long long v, long long* g, long long* hlc3) {
  const long long sv = (long long)v;
  const long long gg = (sv << 43) >> 43;  // sign-extend bits 0..20
  const unsigned long long rest = (unsigned long long)(sv - gg) >> 21;
  const long long hl = (long long)(rest & ((1ull << 21) - 1));
  const long long c3 = (long long)(rest >> 21);
  *g = gg;
  *hlc3 = hl | (c3 << 32);
}

// 32 4-bit bins (one 16-byte chunk of a packed row: feature 2k in the low nibble of byte
// k, 2k + 1 in the high nibble) -> the same bins one per byte (two 16-byte chunks).
__device__ __forceinline__ void unpack4(const uint4 p, uint4& a, uint4& b) {
  const uint32_t in[4] = {p.x, p.y, p.z, p.w};
  uint32_t o[8];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t lo = in[k] & 0x0f0f0f0fu, hi = (in[k] >> 4) & 0x0f0f0f0fu;
    o[2 * k] = __byte_perm(lo, hi, 0x5140);
    o[2 * k + 1] = __byte_perm(lo, hi, 0x7362);
  }
  a = make_uint4(o[0], o[1], o[2], o[3]);
  b = make_uint4(o[4], o[5], o[6], o[7]);
}

// The first NCH 16-feature chunks of a row as one byte per bin: loaded as they are, or
// (PACK4) from half as many packed chunks.
template <int NCH, bool PACK4>
__device__ __forceinline__ void load_row(const uint8_t* __restrict__ row, uint4 (&w)[NCH]) {
  const uint4* rp = reinterpret_cast<const uint4*>(row);
  if (!PACK4) {
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch) w[ch] = rp[ch];
  } else {
#pragma unroll
    for (int pc = 0; pc < (NCH + 1) / 2; ++pc) {
      uint4 a, b;
      unpack4(rp[pc], a, b);
      w[2 * pc] = a;
      if (2 * pc + 1 < NCH) w[2 * pc + 1] = b;
    }
  }
}

template <int MODE>
__device__ __forceinline__ void build_block(const uint8_t* __restrict__ bins, int32_t stride,
                                            bool packed4,
                                            const uint32_t* __restrict__ idx, int32_t begin,
                                            int32_t r0, int32_t r1, bool identity,
                                            const void* __restrict__ gh, const DevGhParams& p,
                                            const DevFeatureGroup& grp,
                                            const int32_t* s_binoff, const uint8_t* s_used,
                                            const long long* s_lut_g, const long long* s_lut_h,
                                            unsigned long long* acc) {
  constexpr int kWords = MODE == GH_QPACK ? 1 : 2;
  const int nf = grp.f_end - grp.f_begin;
  const int nchunks = (nf + 15) >> 4;
  for (int32_t k = r0 + (int32_t)threadIdx.x; k < r1; k += (int32_t)blockDim.x) {
    const uint32_t row = identity ? (uint32_t)(begin + k) : idx[begin + k];
    GhValue<MODE> v;
    v.load(gh, row, p, s_lut_g, s_lut_h);
    const uint8_t* rp = bins + (size_t)row * stride + (packed4 ? grp.f_begin / 2 : grp.f_begin);
    for (int c = 0; c < nchunks; ++c) {
      uint4 w;
      if (packed4) {  // 16 features = half of a packed 16-byte chunk
        uint4 a, b;
        unpack4(*reinterpret_cast<const uint4*>(rp + 16 * (c >> 1)), a, b);
        w = (c & 1) ? b : a;
      } else {
        w = *reinterpret_cast<const uint4*>(rp + 16 * c);
      }
      const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int fl = 16 * c + j;
        if (fl >= nf) break;
        if (!s_used[fl]) continue;
        const uint32_t bin = (words[j >> 2] >> (8 * (j & 3))) & 0xffu;
        unsigned long long* cell = acc + (size_t)kWords * (s_binoff[fl] + bin);
        atomicAdd(cell, (unsigned long long)v.a);
        if (kWords == 2) atomicAdd(cell + 1, (unsigned long long)v.b);
      }
    }
  }
}

template <int MODE>
__device__ __forceinline__ void build_body(const GrowDev& d, int phase) {
  extern __shared__ unsigned long long acc[];
  __shared__ int32_t s_binoff[128];
  __shared__ uint8_t s_used[128];
  __shared__ long long s_lut[MODE == GH_QLUT ? 512 : 1];
  const BuildTarget t = build_target(d, phase);
  build_account(d, phase, t);
  if (!t.ok) return;
  const int32_t begin = t.begin;
  const int32_t count = t.count;
  const int32_t buf = t.buf;
  const DevFeatureGroup grp = d.groups[blockIdx.y];
  const int nf = grp.f_end - grp.f_begin;
  int nb_active = (count + kMinRowsPerBlock - 1) / kMinRowsPerBlock;
  if (nb_active > (int)gridDim.x) nb_active = gridDim.x;
  if (nb_active < 1) nb_active = 1;
  // QPACK field widths hold at most 2^18 rows per CTA.
  if (MODE == GH_QPACK) {
    const int need = (count + (1 << 18) - 1) >> 18;
    if (nb_active < need) nb_active = need;
  }
  if ((int)blockIdx.x >= nb_active) return;
  const int32_t per = (count + nb_active - 1) / nb_active;
  const int32_t r0 = per * (int32_t)blockIdx.x;
  const int32_t r1 = min(count, r0 + per);
  if (r0 >= r1) return;

  constexpr int kWords = MODE == GH_QPACK ? 1 : 2;
  const int nwords = kWords * grp.num_bins;
  for (int i = threadIdx.x; i < nwords; i += blockDim.x) acc[i] = 0ull;
  // Features the parent could not split are neither built nor scanned
  // (learner.rs:2003-2020 build mask).
  {
    const bool sub = t.mask_leaf >= 0;
    const uint8_t* ps = d.splittable + (size_t)(sub ? t.mask_leaf : 0) * d.F;
    for (int fl = threadIdx.x; fl < nf; fl += blockDim.x)
      // feature slices: other ranks own most features and this rank's flags of them are
      // stale, so every feature is accumulated for the ranks that scan it
      s_used[fl] = (sub && !d.sliced) ? ps[grp.f_begin + fl] : (uint8_t)1;
  }
  for (int fl = threadIdx.x; fl < nf; fl += blockDim.x)
    s_binoff[fl] = d.feat[grp.f_begin + fl].bin_off - grp.bin_base;
  if (MODE == GH_QLUT)
    for (int i = threadIdx.x; i < 512; i += blockDim.x)
      s_lut[i] = i < 256 ? d.ghp->lut_g[i] : d.ghp->lut_h[i - 256];
  __syncthreads();
  const DevGhParams& p = *d.ghp;
  const uint32_t* idx = buf == 1 ? d.idx1 : d.idx0;
  build_block<MODE>(d.bins, d.stride, d.packed4 != 0, idx, begin, r0, r1, buf == 2, d.gh, p, grp,
                    s_binoff,
                    s_used, s_lut, s_lut + 256, acc);
  __syncthreads();
  long long* raw = d.raw + 2 * (size_t)grp.bin_base;
  for (int w = threadIdx.x; w < grp.num_bins; w += blockDim.x) {
    if (MODE == GH_QPACK) {
      const unsigned long long v = acc[w];
      if (v) {
        long long g, h;
        unpack_qpack(v, &g, &h);
        if (g) atomicAdd((unsigned long long*)&raw[2 * w], (unsigned long long)g);
        if (h) atomicAdd((unsigned long long*)&raw[2 * w + 1], (unsigned long long)h);
      }
    } else {
      const unsigned long long a = acc[2 * w], b = acc[2 * w + 1];
      if (a) atomicAdd((unsigned long long*)&raw[2 * w], a);
      if (b) atomicAdd((unsigned long long*)&raw[2 * w + 1], b);
    }
  }
}

template <int MODE>
__global__ void __launch_bounds__(kBuildThreads) k_build(GrowDev d, int phase) {
  const SpanStamp span(d);
  build_body<MODE>(d, phase);
  producer_signal(d);
}

// ------------------------------------------------------------------------------------
// Histogram build for quantized gradients with num_grad_quant_bins <= 4 (levels
// qg in [-2,2], qh in [0,4]). One native 32-bit shared atomic per (row, feature)
// adds the signed packed word qg + (qh << 16); rows with qh == 3 (the one level
// that is not a multiple of level 1 after dequantization) also bump a counter that
// sits at a fixed offset from the packed cell. Packed words are folded into 32-bit
// cold sums every kQ4Chunk rows, before a field can overflow.
// Shared-memory cell = (local feature << SHIFT) + bin; SHIFT and the number of
// 16-feature chunks NCH are compile-time so cell offsets fold into immediates.
// Layout (u32 words): hot[kQ4MaxCells] | c3[kQ4MaxCells] | cold_g | cold_q.
// ------------------------------------------------------------------------------------

constexpr int kQ4Threads = 512;
constexpr int kQ4Chunk = 8191;  // |sum qg| <= 2*8191 and sum qh <= 4*8191 fit 16-bit fields

// MASKED: per-feature build mask on every chunk. Otherwise every feature of the group
// is used and only the last chunk (features nf-16(NCH-1) .. 15 absent) is masked.
// AGG (measured, not the default): warp-aggregated atomics. The lanes that hold the same
// bin of a feature are found with __match_any_sync, their packed words summed with
// __reduce_add_sync over that group, and only the group's lowest lane adds the sum (and the
// group's level-3 count). Sums of the same rows: the packed fields fold as before.
template <int SHIFT, int NCH, bool MASKED, bool AGG = false>
__device__ __forceinline__ void q4_row_regs(const uint4 (&w)[NCH], int32_t pv, bool is3,
                                            uint32_t* hot, const uint32_t* mask, uint32_t tail) {
#pragma unroll
  for (int ch = 0; ch < NCH; ++ch) {
    const uint32_t words[4] = {w[ch].x, w[ch].y, w[ch].z, w[ch].w};
    const uint32_t m16 = MASKED ? ((mask[ch >> 1] >> ((ch & 1) * 16)) & 0xffffu) : tail;
    const bool test = MASKED || ch == NCH - 1;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (test && !((m16 >> j) & 1u)) continue;
      const uint32_t bin = (words[j >> 2] >> (8 * (j & 3))) & 0xffu;
      uint32_t* cell = hot + ((16 * ch + j) << SHIFT) + bin;
      if (AGG) {
        const unsigned am = __activemask();
        const unsigned grp = __match_any_sync(am, bin);
        const int sum = __reduce_add_sync(grp, pv);
        const unsigned n3 = (unsigned)__popc(__ballot_sync(am, is3) & grp);
        if ((int)(threadIdx.x & 31) == __ffs(grp) - 1) {
          atomicAdd(reinterpret_cast<int*>(cell), sum);
          if (n3) atomicAdd(cell + kQ4MaxCells, n3);
        }
      } else {
        atomicAdd(reinterpret_cast<int*>(cell), pv);
        if (is3) atomicAdd(cell + kQ4MaxCells, 1u);
      }
    }
  }
}

template <int SHIFT, int NCH, bool MASKED, bool PACK4, bool AGG = false>
__device__ __forceinline__ void q4_row(const uint8_t* __restrict__ rp, int32_t pv, bool is3,
                                       uint32_t* hot, const uint32_t* mask, uint32_t tail) {
  uint4 w[NCH];
  load_row<NCH, PACK4>(rp, w);
  q4_row_regs<SHIFT, NCH, MASKED, AGG>(w, pv, is3, hot, mask, tail);
}

// Build mask of one 128-feature group as four 32-bit words, and whether every feature of
// the group is used (then only the last 16-feature chunk needs a mask: `tail`).
struct Q4Mask {
  uint32_t w[4];
  uint32_t tail;
  bool full;
};

template <int NCH>
__device__ __forceinline__ Q4Mask q4_mask(const uint32_t* s_mask, int nf) {
  Q4Mask m;
#pragma unroll
  for (int i = 0; i < 4; ++i) m.w[i] = s_mask[i];
  const int ntail = nf - 16 * (NCH - 1);  // features in the last chunk, 1..16
  // a short last group (ntail <= 0) never takes the unmasked path: its earlier chunks
  // are incomplete, so `full` below is false
  m.tail = ntail >= 16 ? 0xffffu : (ntail <= 0 ? 0u : ((1u << ntail) - 1u));
  m.full = true;
#pragma unroll
  for (int ch = 0; ch < NCH; ++ch) {
    const uint32_t want = ch == NCH - 1 ? m.tail : 0xffffu;
    const uint32_t m16 = (m.w[ch >> 1] >> ((ch & 1) * 16)) & 0xffffu;
    if (m16 != want) m.full = false;
  }
  return m;
}

template <int SHIFT, int NCH, bool PACK4, bool AGG>
__device__ __forceinline__ void build_q4_body(const GrowDev& d, int phase) {
  extern __shared__ uint32_t sm[];
  __shared__ uint32_t s_mask[4];
  const BuildTarget t = build_target(d, phase);
  build_account(d, phase, t);
  if (!t.ok) return;
  const int32_t begin = t.begin;
  const int32_t count = t.count;
  const int32_t buf = t.buf;
  const DevFeatureGroup grp = d.groups[blockIdx.y];
  const int nf = grp.f_end - grp.f_begin;
  const int cap = nf << SHIFT;  // <= kQ4MaxCells (host group planning)
  int nb_active = (count + kMinRowsPerBlock - 1) / kMinRowsPerBlock;
  if (nb_active > (int)gridDim.x) nb_active = gridDim.x;
  if (nb_active < 1) nb_active = 1;
  if ((int)blockIdx.x >= nb_active) return;
  const int32_t per = (count + nb_active - 1) / nb_active;  // <= 65535 (host grid sizing)
  const int32_t r0 = per * (int32_t)blockIdx.x;
  const int32_t r1 = min(count, r0 + per);
  if (r0 >= r1) return;

  uint32_t* hot = sm;
  uint32_t* c3 = sm + kQ4MaxCells;
  int32_t* cold_g = reinterpret_cast<int32_t*>(sm + 2 * kQ4MaxCells);
  int32_t* cold_q = reinterpret_cast<int32_t*>(sm + 3 * kQ4MaxCells);
  // cold sums exist only when this CTA's range needs more than one chunk
  const bool folds = (r1 - r0) > kQ4Chunk;
  {
    uint4* h4 = reinterpret_cast<uint4*>(hot);
    uint4* c4 = reinterpret_cast<uint4*>(c3);
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
    for (int i = threadIdx.x; i < (cap + 3) / 4; i += kQ4Threads) {
      h4[i] = z;
      c4[i] = z;
    }
    if (folds) {
      uint4* g4 = reinterpret_cast<uint4*>(cold_g);
      uint4* q4 = reinterpret_cast<uint4*>(cold_q);
      for (int i = threadIdx.x; i < (cap + 3) / 4; i += kQ4Threads) {
        g4[i] = z;
        q4[i] = z;
      }
    }
  }
  // Features the parent could not split are neither built nor scanned
  // (learner.rs:2003-2020 build mask).
  const bool sub = t.mask_leaf >= 0;
  const uint8_t* ps = d.splittable + (size_t)(sub ? t.mask_leaf : 0) * d.F + grp.f_begin;
  if (threadIdx.x < 128) {
    const int fl = threadIdx.x;
    const uint32_t m =
        __ballot_sync(0xffffffffu, fl < nf && (!sub || d.sliced || ps[fl] != 0));
    if ((fl & 31) == 0) s_mask[fl >> 5] = m;
  }
  __syncthreads();
  const Q4Mask qm = q4_mask<NCH>(s_mask, nf);
  const uint32_t* mask = qm.w;
  const uint32_t tail = qm.tail;
  const bool full = qm.full;
  const uint32_t* idx = buf == 1 ? d.idx1 : d.idx0;
  const uint16_t* gq = reinterpret_cast<const uint16_t*>(d.gh);
  const bool identity = buf == 2;
  const uint8_t* bins = d.bins + (PACK4 ? grp.f_begin / 2 : grp.f_begin);
  const size_t stride = (size_t)d.stride;
  for (int32_t cs = r0; cs < r1; cs += kQ4Chunk) {
    const int32_t ce = min(r1, cs + kQ4Chunk);
    for (int32_t k = cs + (int32_t)threadIdx.x; k < ce; k += 2 * kQ4Threads) {
      const int32_t k2 = k + kQ4Threads;
      const bool two = k2 < ce;
      const uint32_t row0 = identity ? (uint32_t)(begin + k) : idx[begin + k];
      const uint32_t row1 = two ? (identity ? (uint32_t)(begin + k2) : idx[begin + k2]) : row0;
      const uint16_t q0 = gq[row0];
      const uint16_t q1 = gq[row1];
      const uint8_t* rp0 = bins + (size_t)row0 * stride;
      const uint8_t* rp1 = bins + (size_t)row1 * stride;
      const int qg0 = (int)(int8_t)(q0 & 0xff), qh0 = (int)(int8_t)(q0 >> 8);
      const int qg1 = (int)(int8_t)(q1 & 0xff), qh1 = (int)(int8_t)(q1 >> 8);
      if (full) {
        q4_row<SHIFT, NCH, false, PACK4, AGG>(rp0, qg0 + (qh0 << 16), qh0 == 3, hot, mask, tail);
        if (two)
          q4_row<SHIFT, NCH, false, PACK4, AGG>(rp1, qg1 + (qh1 << 16), qh1 == 3, hot, mask,
                                                tail);
      } else {
        q4_row<SHIFT, NCH, true, PACK4, AGG>(rp0, qg0 + (qh0 << 16), qh0 == 3, hot, mask, tail);
        if (two)
          q4_row<SHIFT, NCH, true, PACK4, AGG>(rp1, qg1 + (qh1 << 16), qh1 == 3, hot, mask,
                                               tail);
      }
    }
    if (ce < r1) {
      __syncthreads();
      for (int s = threadIdx.x; s < cap; s += kQ4Threads) {
        const int32_t v = (int32_t)hot[s];
        const int32_t lo = (int32_t)(int16_t)(v & 0xffff);
        cold_g[s] += lo;
        cold_q[s] += (v - lo) >> 16;
        hot[s] = 0u;
      }
      __syncthreads();
    }
  }
  __syncthreads();
  long long* raw = d.raw;
  for (int s = threadIdx.x; s < cap; s += kQ4Threads) {
    const int fl = s >> SHIFT;
    const int bin = s & ((1 << SHIFT) - 1);
    if (fl >= nf) continue;
    // feature tables are read from global memory here: with no static shared arrays the
    // CTA's shared footprint lets two CTAs share an SM
    const DevFeature* fp = d.feat + grp.f_begin + fl;
    if (bin >= __ldg(&fp->num_bin)) continue;
    const int32_t v = (int32_t)hot[s];
    const int32_t lo = (int32_t)(int16_t)(v & 0xffff);
    const long long g = (folds ? (long long)cold_g[s] : 0ll) + lo;
    const long long qsum = (folds ? (long long)cold_q[s] : 0ll) + ((v - lo) >> 16);
    const long long n3 = (long long)c3[s];
    const long long h = (qsum - 3 * n3) | (n3 << 32);
    const size_t gb = (size_t)(__ldg(&fp->bin_off) + bin);
    if (g) atomicAdd(reinterpret_cast<unsigned long long*>(&raw[2 * gb]), (unsigned long long)g);
    if (h)
      atomicAdd(reinterpret_cast<unsigned long long*>(&raw[2 * gb + 1]), (unsigned long long)h);
  }
}

template <int SHIFT, int NCH, bool PACK4 = false, bool AGG = false>
__global__ void __launch_bounds__(kQ4Threads, 2) k_build_q4(GrowDev d, int phase) {
  const SpanStamp span(d);
  build_q4_body<SHIFT, NCH, PACK4, AGG>(d, phase);
  producer_signal(d);
}

// (SHIFT, NCH) instantiations with (16 * (NCH - 1) + 1) << SHIFT <= kQ4MaxCells.
using Q4Kernel = void (*)(GrowDev, int);
__host__ Q4Kernel q4_kernel(int shift, int nch, bool pack4 = false, bool agg = false) {
  // warp-aggregated atomics: one instantiation, the C1 layout (measured, not the default)
  if (agg && !pack4 && shift == 8 && nch == 2) return k_build_q4<8, 2, false, true>;
  if (pack4) {  // 4-bit rows: every feature has at most 16 bins (shift 4)
#define Q4P_CASE(N) \
  if (shift == 4 && nch == N) return k_build_q4<4, N, true>;
    Q4P_CASE(1) Q4P_CASE(2) Q4P_CASE(3) Q4P_CASE(4) Q4P_CASE(5) Q4P_CASE(6) Q4P_CASE(7)
    Q4P_CASE(8)
#undef Q4P_CASE
    return nullptr;
  }
#define Q4_CASE(S, N) \
  if (shift == S && nch == N) return k_build_q4<S, N>;
  Q4_CASE(4, 1) Q4_CASE(4, 2) Q4_CASE(4, 3) Q4_CASE(4, 4)
  Q4_CASE(4, 5) Q4_CASE(4, 6) Q4_CASE(4, 7) Q4_CASE(4, 8)
  Q4_CASE(5, 1) Q4_CASE(5, 2) Q4_CASE(5, 3) Q4_CASE(5, 4)
  Q4_CASE(5, 5) Q4_CASE(5, 6) Q4_CASE(5, 7) Q4_CASE(5, 8)
  Q4_CASE(6, 1) Q4_CASE(6, 2) Q4_CASE(6, 3) Q4_CASE(6, 4)
  Q4_CASE(6, 5) Q4_CASE(6, 6) Q4_CASE(6, 7)
  Q4_CASE(7, 1) Q4_CASE(7, 2) Q4_CASE(7, 3) Q4_CASE(7, 4)
  Q4_CASE(8, 1) Q4_CASE(8, 2)
#undef Q4_CASE
  return nullptr;
}

// ------------------------------------------------------------------------------------
// Threshold scan of one direction of one feature by one warp
// (find_best_split_cpu_native, lgbm-compute/src/kernels/split.rs:8970-9329).
// The dependent f64 chains (running gradient / hessian sums, seeded with kEpsilon)
// run sequentially in one lane each, in the reference's order; the integer count
// prefix and the per-candidate gains run across the warp.
// ------------------------------------------------------------------------------------

struct ScanCand {
  int32_t has;         // a candidate cleared min_gain_shift (is_splittable)
  int32_t best_k;      // -1 if none
  double gain;
  double slg, slh;
  int32_t lc;
  int32_t thr;
};

struct ScanLeaf {
  double sum_g, sum_h, parent_output;
  int32_t num_data;
};

// Named barrier over one G-thread group (ids 1..15; id 0 is __syncthreads).
template <int G = 256>
__device__ __forceinline__ void group_sync(int id) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(G) : "memory");
}

// p[k] <- init + p[0] + ... + p[k] in place, strictly left to right: the reference's
// sequential f64 accumulation. Blocks of 16 addends are loaded into registers first,
// so each step costs one dependent add.
__device__ __forceinline__ double seq_prefix_inplace(double* p, int count, double init) {
  double acc = init;
  int k = 0;
  for (; k + 16 <= count; k += 16) {
    double v[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = p[k + j];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      acc += v[j];
      v[j] = acc;
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) p[k + j] = v[j];
  }
  for (; k < count; ++k) {
    acc += p[k];
    p[k] = acc;
  }
  return acc;
}

// init - v[0] - v[stride] - ... - v[(n-1)*stride], strictly left to right.
__device__ __forceinline__ double seq_sub(const double* v, int stride, int n, double init) {
  double acc = init;
  int k = 0;
  for (; k + 16 <= n; k += 16) {
    double x[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) x[j] = v[(k + j) * stride];
#pragma unroll
    for (int j = 0; j < 16; ++j) acc -= x[j];
  }
  for (; k < n; ++k) acc -= v[k * stride];
  return acc;
}

// Asynchronous prefetch of [p, p + bytes) into L2 (p and bytes multiples of 16).
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v)
               : "memory");
  return old;
}

__device__ __forceinline__ void warp_best(double& gain, int32_t& k) {
  // max gain, ties to the smallest k (first in scan order)
  for (int o = 16; o > 0; o >>= 1) {
    const double og = __shfl_xor_sync(0xffffffffu, gain, o);
    const int32_t ok = __shfl_xor_sync(0xffffffffu, k, o);
    if (og > gain || (og == gain && ok >= 0 && (k < 0 || ok < k))) {
      gain = og;
      k = ok;
    }
  }
}

constexpr int kScanGroup = 256;  // threads per (leaf, direction) scan: one candidate each

struct ScanScratch {
  double pg[kMaxBins];   // addends, then running gradient sums
  double ph[kMaxBins];   // addends, then running hessian sums
  int32_t pc[kMaxBins];  // running counts
  int32_t wsum[8];
  int32_t wpre[8];
  int32_t wmin[8];
  int32_t wk[8];
  int32_t whas[8];
  double wgain[8];
};

// One direction of find_best_split_cpu_native (lgbm-compute/src/kernels/split.rs:8970-9329)
// for one feature, by one G-thread group (thread k owns candidate step k). The two
// dependent f64 chains (running gradient and hessian sums, the hessian seeded with
// kEpsilon) run sequentially in the reference's order on threads 0 and 32; counts,
// the sticky stop, gains and the first-max selection run across the group.
template <int G>
__device__ void scan_direction(const double* hist, const DevFeature& f, const DevGainConfig& cfg,
                               const ScanLeaf& leaf, bool forward, ScanScratch& s, int bar_id,
                               ScanCand* out) {
  const int gt = threadIdx.x & (G - 1);
  const int lane = gt & 31, wg = gt >> 5;
  const double eps = k_eps();
  const int nb = f.num_bin;
  const int offset = f.offset;
  const int na = (f.flags & 2) ? 1 : 0;
  const bool skip_def = (f.flags & 1) != 0;
  const double bumped = leaf.sum_h + 2.0 * eps;
  const double cnt_factor = (double)leaf.num_data / bumped;
  const int32_t min_data = cfg.min_data_in_leaf;
  const double min_hess = cfg.min_sum_hessian_in_leaf;
  int count, t0;  // t = forward ? t0 + k : t0 - k
  bool na_pre = false;
  if (!forward) {
    count = max(nb - 1 - na, 0);
    t0 = nb - 1 - offset - na;
  } else {
    na_pre = na && offset == 1;
    count = (f.flags & 4) ? max(nb - 1 - offset, 0) + (na_pre ? 1 : 0) : 0;
    t0 = na_pre ? -1 : 0;
    if (count == 0) na_pre = false;
  }
  // 1. addend of step k (0 when the step is inactive; the running sums are never -0.0,
  //    so `+ 0.0` leaves them unchanged, split.rs:8950-8960)
  const int k = gt;
  const int t = forward ? t0 + k : t0 - k;
  const bool skip = skip_def && (t + offset) == f.default_bin;
  const bool act = k < count && (forward ? !skip : (t >= (1 - offset) && !skip));
  const bool act_t = act && t >= 0;
  const double ah = act_t ? hist[2 * t + 1] : 0.0;
  if (k < count) {
    s.pg[k] = act_t ? hist[2 * t] : 0.0;
    s.ph[k] = ah;
  }
  int32_t cv = act_t ? d_round_int(ah * cnt_factor) : 0;
  int32_t pre = (na_pre && gt < nb - offset) ? d_round_int(hist[2 * gt + 1] * cnt_factor) : 0;
  group_sync<G>(bar_id);
  // 2. sequential chains
  if ((gt == 0 || gt == 32) && count > 0) {
    const bool isg = gt == 0;
    double init = isg ? 0.0 : eps;
    if (na_pre)  // NA preamble (split.rs:9183-9199): leaf totals minus every explicit bin
      init = isg ? seq_sub(hist, 2, nb - offset, leaf.sum_g)
                 : seq_sub(hist + 1, 2, nb - offset, bumped - eps);
    seq_prefix_inplace(isg ? s.pg : s.ph, count, init);
  }
  // 3. integer count prefix across the group
  int32_t incl = cv;
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  for (int o = 16; o > 0; o >>= 1) pre += __shfl_xor_sync(0xffffffffu, pre, o);
  if (lane == 31) s.wsum[wg] = incl;
  if (lane == 0) s.wpre[wg] = pre;
  group_sync<G>(bar_id);
  int32_t c_init = 0, woff = 0;
  if (na_pre) {
    int32_t tot = 0;
#pragma unroll
    for (int w = 0; w < G / 32; ++w) tot += s.wpre[w];
    c_init = leaf.num_data - tot;
  }
#pragma unroll
  for (int w = 0; w < G / 32; ++w)
    if (w < wg) woff += s.wsum[w];
  const int32_t c_own = c_init + woff + incl;
  const int32_t c_oth = leaf.num_data - c_own;
  double g_own = 0.0, h_own = 0.0;
  if (k < count) {
    g_own = s.pg[k];
    h_own = s.ph[k];
    s.pc[k] = c_own;
  }
  const double h_oth = bumped - h_own;
  const bool cont = c_own < min_data || h_own < min_hess;
  const bool brk = c_oth < min_data || h_oth < min_hess;
  // 4. first step that breaks the scan (sticky `done`)
  int32_t kst = (act && !cont && brk) ? k : 0x7fffffff;
  for (int o = 16; o > 0; o >>= 1) kst = min(kst, __shfl_xor_sync(0xffffffffu, kst, o));
  if (lane == 0) s.wmin[wg] = kst;
  group_sync<G>(bar_id);
  int32_t kstar = 0x7fffffff;
#pragma unroll
  for (int w = 0; w < G / 32; ++w) kstar = min(kstar, s.wmin[w]);
  // 5. candidate gain of step k
  double best_gain = kNegInf;
  int32_t best_k = -1;
  int32_t has = 0;
  if (act && !cont && k < kstar) {
    const double gain_shift = d_leaf_gain_full(cfg, leaf.sum_g, bumped, leaf.num_data,
                                               leaf.parent_output);
    const double min_gain_shift = gain_shift + cfg.min_gain_to_split;
    const double g_oth = leaf.sum_g - g_own;
    double gain;
    if (!forward)  // own side is the right child
      gain = d_split_gain(cfg, g_oth, h_oth, g_own, h_own, c_oth, c_own, leaf.parent_output);
    else
      gain = d_split_gain(cfg, g_own, h_own, g_oth, h_oth, c_own, c_oth, leaf.parent_output);
    if (gain > min_gain_shift) {
      has = 1;
      best_gain = gain;
      best_k = k;
    }
  }
  has = __any_sync(0xffffffffu, has) ? 1 : 0;
  warp_best(best_gain, best_k);
  if (lane == 0) {
    s.wgain[wg] = best_gain;
    s.wk[wg] = best_k;
    s.whas[wg] = has;
  }
  group_sync<G>(bar_id);
  if (gt == 0) {
    double bg = kNegInf;
    int32_t bk = -1, hs = 0;
#pragma unroll
    for (int w = 0; w < G / 32; ++w) {
      hs |= s.whas[w];
      const double g = s.wgain[w];
      const int32_t kk = s.wk[w];
      if (g > bg || (g == bg && kk >= 0 && (bk < 0 || kk < bk))) {
        bg = g;
        bk = kk;
      }
    }
    out->has = hs;
    out->best_k = bk;
    out->gain = bg;
    if (bk >= 0) {
      const int tb = forward ? t0 + bk : t0 - bk;
      if (!forward) {
        out->slg = leaf.sum_g - s.pg[bk];
        out->slh = bumped - s.ph[bk];
        out->lc = leaf.num_data - s.pc[bk];
        out->thr = tb - 1 + offset;
      } else {
        out->slg = s.pg[bk];
        out->slh = s.ph[bk];
        out->lc = s.pc[bk];
        out->thr = tb + offset;
      }
    }
  }
}

// Finalization of the winning candidate (split.rs:9267-9326).
__device__ DevSplitInfo finalize_split(const DevGainConfig& cfg, const ScanLeaf& leaf,
                                       const ScanCand& rev, const ScanCand& fwd) {
  const double eps = k_eps();
  const double bumped = leaf.sum_h + 2.0 * eps;
  const double min_gain_shift =
      d_leaf_gain_full(cfg, leaf.sum_g, bumped, leaf.num_data, leaf.parent_output) +
      cfg.min_gain_to_split;
  bool splittable = rev.has || fwd.has;
  double best_gain = kNegInf;
  double slg = 0.0, slh = 0.0;
  int32_t lc = 0, thr = 0, dl = 1;
  if (rev.best_k >= 0) {
    best_gain = rev.gain;
    slg = rev.slg;
    slh = rev.slh;
    lc = rev.lc;
    thr = rev.thr;
    dl = 1;
  }
  if (fwd.best_k >= 0 && fwd.gain > best_gain) {
    best_gain = fwd.gain;
    slg = fwd.slg;
    slh = fwd.slh;
    lc = fwd.lc;
    thr = fwd.thr;
    dl = 0;
  }
  if (!(splittable && best_gain > kNegInf)) return d_split_none();
  DevSplitInfo s;
  const int32_t rc = leaf.num_data - lc;
  s.threshold = (uint32_t)thr;
  s.default_left = dl;
  s.left_count = lc;
  s.right_count = rc;
  s.gain = best_gain - min_gain_shift;
  s.left_sum_gradient = slg;
  s.left_sum_hessian = slh - eps;
  const double rsg = leaf.sum_g - slg;
  const double rsh = bumped - slh;
  s.right_sum_gradient = rsg;
  s.right_sum_hessian = rsh - eps;
  s.left_output = d_leaf_output_full(cfg, cfg.use_smoothing, slg, slh, lc, leaf.parent_output);
  s.right_output = d_leaf_output_full(cfg, cfg.use_smoothing, rsg, rsh, rc, leaf.parent_output);
  return s;
}

// ------------------------------------------------------------------------------------
// Per-split control kernel.
// ------------------------------------------------------------------------------------

__global__ void k_tree_init(GrowDev d) {
  GrowCtrl* c = d.ctrl;
  const bool stopped = d.stopped && *d.stopped;
  const int gtid = blockIdx.x * blockDim.x + threadIdx.x;
  const int gsz = gridDim.x * blockDim.x;
  for (int l = gtid; l < d.L; l += gsz) {
    d.leaf_begin[l] = 0;
    d.leaf_count[l] = 0;
    d.leaf_count_g[l] = 0;
    d.leaf_buf[l] = 0;
    d.slot_of_leaf[l] = -1;
    d.best[l] = d_split_none();
    d.best_feature[l] = -1;
    d.t_left[l] = 0;
    d.t_right[l] = 0;
    d.t_split_feature[l] = 0;
    d.t_threshold[l] = 0;
    d.t_split_gain[l] = 0.f;
    d.t_decision[l] = 0;
    d.t_leaf_value[l] = 0.0;
    d.t_leaf_weight[l] = 0.0;
    d.t_leaf_count[l] = 0;
    d.t_internal_value[l] = 0.0;
    d.t_internal_count[l] = 0;
    d.t_leaf_depth[l] = 0;
    d.t_leaf_parent[l] = 0;
    d.leaf_is_right[l] = 0;
  }
  const size_t nsp = (size_t)d.L * d.F;
  for (size_t i = gtid; i < nsp; i += gsz) d.splittable[i] = 1;
  for (int i = gtid; i < d.max_tiles; i += gsz) d.part_status[i] = 0ull;
  // both peer-exchange accumulators start the tree empty (every rank has finished the
  // previous tree: the gradient step's reductions came in between)
  if (d.xranks > 1)
    for (size_t i = gtid; i < 2 * ((size_t)d.raw_len + 2); i += gsz) d.xlocal[i] = 0;
  // look-ahead slots: empty accumulators, no recorded leaf, no stale status words
  if (d.lookahead) {
    for (size_t i = gtid; i < kLaSlots * ((size_t)d.raw_len + 2); i += gsz) d.la_raw[i] = 0;
    for (int i = gtid; i < d.max_tiles; i += gsz) d.la_status[i] = 0ull;
    if (gtid < kLaSlots) d.la[gtid] = LookAhead{};
  }
  if (gtid == 0) {
    const uint32_t epoch = c->epoch;
    const uint32_t err = c->error;
    GrowCtrl z = {};
    *c = z;
    c->epoch = epoch;
    c->error = err;
    // the tree's look-ahead signals count from here (every earlier one has been sent)
    c->la_base = (d.lookahead && d.xranks > 1) ? *d.la_seq : 0ull;
    c->num_leaves = 1;
    c->left_leaf = 0;
    c->right_leaf = -1;
    c->next_slot = 0;
    d.leaf_count[0] = (int32_t)d.N;
    d.leaf_count_g[0] = (int32_t)d.n_global;
    d.leaf_buf[0] = 2;
    const DevGhParams& p = *d.ghp;
    // LeafSplits::init over all rows (leaf_splits.rs:75-92): integer root sums
    // decoded exactly like histogram cells.
    DevLeafSplits r;
    r.num_data = (int32_t)d.n_global;
    r._pad = 0;
    r.sum_g = decode_g(p, p.root_g);
    r.sum_h = decode_h(p, p.root_h);
    // self_output: max_delta_step clamps, no smoothing (leaf_splits.rs:128-145)
    r.weight = d_leaf_output_full(d.gain, false, r.sum_g, r.sum_h, 0, 0.0);
    d.ls[0] = r;
    d.t_leaf_value[0] = r.weight;
    d.t_leaf_count[0] = (int32_t)d.n_global;
    d.t_leaf_parent[0] = -1;
    if (stopped) c->done = 1;
    if (!(r.sum_h > 0.0)) {
      c->error |= kErrRootHessian;
      c->done = 1;
    }
  }
}

// ------------------------------------------------------------------------------------
// Per-split control step: apply the split chosen at step s-1 (learner.rs:3895-4092),
// BeforeFindBestSplit gates (learner.rs:1808-1839), smaller child and pool slots
// (learner.rs:1882-1916). It runs in thread 0 of every k_fixscan CTA from the same
// inputs (prep_compute only reads), and the kernel's last CTA writes the result
// (prep_commit), after every CTA has read what it needs. Leaf counts come in two kinds:
// rows on this device (ranges of the index buffers) and rows on all devices (tree
// counts, gates, smaller child, LeafSplits); with one device they are equal.
// ------------------------------------------------------------------------------------

struct Prep {
  GrowCtrl c;  // control block after this step
  int32_t main_needed;  // the pending split still needs its main partition (no look-ahead)
  int32_t applied;
  int32_t leaf, nr, node, parent, parent_is_right;
  int32_t lc, rc, lcg, rcg, dst, beg, depth;
  int32_t feature;
  int32_t cat_index;  // categorical node: its index among the tree's categorical nodes
  int8_t dt;
  float split_gain;
  double old_value;
  DevLeafSplits lsL, lsR;  // children (applied)
  int32_t live;            // the two leaves below are scanned
  int32_t kill0, kill1;    // leaves whose best split is cleared by the gates (-1: none)
  int32_t slot_leaf0, slot_val0, slot_leaf1, slot_val1;  // slot_of_leaf writes (-1: none)
  int32_t S, Lg, sslot, lslot, use_sub, mask_leaf, smaller_is_left;
  DevLeafSplits lsS, lsLg;
  int32_t priv_tiles;  // > 0: the accumulated child is this many per-tile partials
  int32_t acc_slot;    // >= 0: the pending split was partitioned by this look-ahead slot
  int32_t la_clear;    // >= 0: the look-ahead slot this step clears (look-ahead on)
};

template <bool PEER>
__device__ void prep_compute(const GrowDev& d, int s, Prep& P) {
  // the control block is updated in place in P (shared memory in the control step)
  GrowCtrl& c = P.c;
  c = *d.ctrl;
  P.main_needed = (!c.done && c.pending && !c.pend_la) ? 1 : 0;
  P.applied = 0;
  P.live = 0;
  P.kill0 = P.kill1 = -1;
  P.slot_leaf0 = P.slot_leaf1 = -1;
  P.slot_val0 = P.slot_val1 = -1;
  P.S = P.Lg = -1;
  P.sslot = P.lslot = -1;
  P.use_sub = 0;
  P.mask_leaf = -1;
  P.smaller_is_left = 1;
  P.priv_tiles = 0;
  P.acc_slot = -1;
  P.la_clear = -1;
  // Look-aheads of this tree that have finished (this step waited for the one of step
  // s - 2): the one of step s - 3 is counted and its slot cleared here (every rank has
  // consumed it by now); the one of step s - 2 is consumed when step s - 1 picked its leaf
  // (the final step also counts it: no later step will).
  const LookAhead* lar = nullptr;
  if (d.lookahead) {
    constexpr int M = kLaSlots - 1;
    P.la_clear = (s + 1) & M;
    auto count_la = [&](const LookAhead& r) {
      if (r.active && r.ran) {
        c.la_runs += 1;
        c.la_rows += r.rows;
      }
      if (r.failed) {
        c.error |= kErrSpinTimeout;
        c.done = 1;
      }
    };
    if (s >= 3) count_la(d.la[(s + 1) & M]);
    if (s >= 2 && s == d.L - 1) count_la(d.la[(s + 2) & M]);
    if (s >= 2 && c.pending && c.pend_la == 1 + ((s + 2) & M)) {
      const LookAhead& r = d.la[(s + 2) & M];
      lar = &r;
      P.acc_slot = (s + 2) & M;
      c.la_hits += 1;
      c.rows_parted += r.rows;
      if (r.build) {
        c.rows_built += r.built;
        c.num_builds += 1;
      }
    }
  }
  int32_t left = c.left_leaf, right = c.right_leaf;
  int32_t cnt_left = 0, cnt_right = 0, depth_left = 0, slot_left = -1;
  bool known = false;
  DevLeafSplits lsL{}, lsR{};
  if (c.pending) {
    const int32_t leaf = c.split_leaf;
    const int32_t nr = c.num_leaves;
    const int32_t f = c.split_feature;
    const DevSplitInfo b = c.split;
    const int32_t cnt = d.leaf_count[leaf];
    const int32_t cntg = d.leaf_count_g[leaf];
    const int32_t beg = d.leaf_begin[leaf];
    const int32_t src = d.leaf_buf[leaf];
    const int32_t parent = d.t_leaf_parent[leaf];
    const double old_value = d.t_leaf_value[leaf];
    const int32_t depth = d.t_leaf_depth[leaf];
    const int32_t mt = d.feat[f].missing_type;
    // the look-ahead's left rows: this device's, summed over the devices with several
    const long long lcg_raw = lar ? (PEER ? la_sum<PEER>(d, P.acc_slot, (size_t)d.raw_len)
                                          : (long long)lar->left_total)
                                  : raw_sum<PEER>(d, (size_t)d.raw_len);
    slot_left = d.slot_of_leaf[leaf];
    // read with the leaf's other fields (the parent's child pointer would be a
    // dependent round trip)
    const int32_t is_right = d.leaf_is_right[leaf];
    const int32_t lc = lar ? lar->left_total : c.part_left_total;
    const int32_t lcg = (int32_t)lcg_raw;
    P.applied = 1;
    P.leaf = leaf;
    P.nr = nr;
    P.node = nr - 1;
    P.parent = parent;
    P.parent_is_right = parent >= 0 && is_right != 0;
    P.lc = lc;
    P.rc = cnt - lc;
    P.lcg = lcg;
    P.rcg = cntg - lcg;
    P.dst = src == 1 ? 0 : 1;
    P.beg = beg;
    P.depth = depth;
    P.feature = f;
    int8_t dt = 0;
    P.cat_index = -1;
    if (d.feat[f].flags & kFeatCategorical) {
      // Tree::split_categorical (lgbm-model/src/tree.rs:710-770): categorical bit, the
      // node's threshold is its categorical-node index, default_left is not encoded
      dt |= 1;
      P.cat_index = c.num_cat;
      c.num_cat += 1;
    } else if (b.default_left) {
      dt |= 2;
    }
    dt |= (int8_t)((mt & 3) << 2);
    P.dt = dt;
    P.split_gain = (float)(b.gain + d.gain.min_gain_to_split);
    P.old_value = old_value;
    // child LeafSplits seeded from the SplitInfo (learner.rs:4061-4089)
    lsL.num_data = lcg;
    lsL._pad = 0;
    lsL.sum_g = b.left_sum_gradient;
    lsL.sum_h = b.left_sum_hessian;
    lsL.weight = b.left_output;
    lsR.num_data = P.rcg;
    lsR._pad = 0;
    lsR.sum_g = b.right_sum_gradient;
    lsR.sum_h = b.right_sum_hessian;
    lsR.weight = b.right_output;
    P.lsL = lsL;
    P.lsR = lsR;
    if (d.fused && d.private_tiles > 0) {
      const int32_t nt = (cnt + kPartitionTileRows - 1) / kPartitionTileRows;
      if (nt <= d.private_tiles) P.priv_tiles = nt;
    }
    left = leaf;
    right = nr;
    cnt_left = lcg;
    cnt_right = P.rcg;
    depth_left = depth + 1;
    known = true;
    c.left_leaf = leaf;
    c.right_leaf = nr;
    c.num_leaves = nr + 1;
    c.num_splits += 1;
    c.pending = 0;
    c.pend_la = 0;
  }
  if (c.done || s >= d.L - 1) {
    c.do_find = 0;
    return;
  }
  if (!known) {
    cnt_left = d.leaf_count_g[left];
    cnt_right = right >= 0 ? d.leaf_count_g[right] : 0;
    depth_left = d.t_leaf_depth[left];
    slot_left = d.slot_of_leaf[left];
    lsL = d.ls[left];
    if (right >= 0) lsR = d.ls[right];
  }
  c.epoch += 1;
  c.part_ticket = 0;
  c.part_left_total = 0;
  c.scan_counter = 0;
  // ---- BeforeFindBestSplit (learner.rs:1808-1839) ----
  const int32_t min2 = d.gain.min_data_in_leaf * 2;
  int32_t did = 1;
  if (d.max_depth > 0 && depth_left >= d.max_depth) {
    P.kill0 = left;
    P.kill1 = right;
    did = 0;
  } else if (right >= 0) {
    if (cnt_right < min2 && cnt_left < min2) {
      P.kill0 = left;
      P.kill1 = right;
      did = 0;
    }
  } else if (cnt_left < min2) {
    P.kill0 = left;
    did = 0;
  }
  c.do_find = did;
  if (!did) {
    return;
  }
  // ---- smaller child + pool slots (learner.rs:1882-1916) ----
  int32_t smaller, larger;
  DevLeafSplits ls_smaller, ls_larger{};
  if (right < 0) {
    smaller = left;
    larger = -1;
    ls_smaller = lsL;
  } else if (cnt_left < cnt_right) {
    smaller = left;
    larger = right;
    ls_smaller = lsL;
    ls_larger = lsR;
  } else {
    smaller = right;
    larger = left;
    ls_smaller = lsR;
    ls_larger = lsL;
  }
  int32_t ss, lsl = -1, use_sub = 0;
  if (right < 0) {
    if (slot_left < 0) {
      slot_left = c.next_slot++;
      P.slot_leaf0 = left;
      P.slot_val0 = slot_left;
    }
    ss = slot_left;
  } else {
    const int32_t parent_slot = slot_left;
    use_sub = parent_slot >= 0 ? 1 : 0;
    ss = c.next_slot++;
    if (smaller == left) {
      P.slot_leaf0 = right;
      P.slot_val0 = parent_slot;
      P.slot_leaf1 = left;
      P.slot_val1 = ss;
    } else {
      P.slot_leaf0 = right;
      P.slot_val0 = ss;
    }
    lsl = parent_slot;
    if (!use_sub) {
      // Cannot happen with a one-slot-per-leaf pool: a leaf is split only after its
      // histogram was built or derived.
      c.error |= kErrNoParentHistogram;
      c.done = 1;
      c.do_find = 0;
      return;
    }
  }
  c.smaller_leaf = smaller;
  c.larger_leaf = larger;
  c.smaller_slot = ss;
  c.larger_slot = lsl;
  c.use_subtract = use_sub;
  P.live = 1;
  P.S = smaller;
  P.Lg = larger;
  P.sslot = ss;
  P.lslot = lsl;
  P.use_sub = use_sub;
  P.mask_leaf = left;  // the leaf that was split keeps the left child's id
  P.smaller_is_left = smaller == left;
  P.lsS = ls_smaller;
  P.lsLg = ls_larger;
}

// Writes of the control step except the control block itself. CAT: the dataset has
// categorical features, whose nodes also record their bin set.
template <bool CAT>
__device__ void prep_commit(const GrowDev& d, const Prep& P) {
  if (P.applied) {
    const int32_t leaf = P.leaf, nr = P.nr, node = P.node;
    const DevSplitInfo& b = P.c.split;
    d.leaf_begin[nr] = P.beg + P.lc;
    d.leaf_count[leaf] = P.lc;
    d.leaf_count[nr] = P.rc;
    d.leaf_count_g[leaf] = P.lcg;
    d.leaf_count_g[nr] = P.rcg;
    d.leaf_buf[leaf] = P.dst;
    d.leaf_buf[nr] = P.dst;
    // Tree::split (lgbm-model/src/tree.rs:614-690)
    if (P.parent >= 0) {
      if (P.parent_is_right)
        d.t_right[P.parent] = node;
      else
        d.t_left[P.parent] = node;
    }
    d.t_split_feature[node] = P.feature;
    d.t_split_gain[node] = P.split_gain;
    d.t_threshold[node] = P.cat_index >= 0 ? (uint32_t)P.cat_index : b.threshold;
    if (CAT)
      for (int k = 0; k < kCatWords; ++k)
        d.t_cat[(size_t)node * kCatWords + k] = P.cat_index >= 0 ? d.split_cat[k] : 0u;
    d.t_internal_value[node] = P.old_value;
    d.t_internal_count[node] = P.lcg + P.rcg;
    d.t_left[node] = ~leaf;
    d.t_right[node] = ~nr;
    d.t_decision[node] = P.dt;
    d.t_leaf_value[leaf] = b.left_output;
    d.t_leaf_weight[leaf] = b.left_sum_hessian;
    d.t_leaf_count[leaf] = P.lcg;
    d.t_leaf_value[nr] = b.right_output;
    d.t_leaf_weight[nr] = b.right_sum_hessian;
    d.t_leaf_count[nr] = P.rcg;
    d.t_leaf_depth[nr] = P.depth + 1;
    d.t_leaf_depth[leaf] = P.depth + 1;
    d.t_leaf_parent[leaf] = node;
    d.t_leaf_parent[nr] = node;
    d.leaf_is_right[leaf] = 0;  // the split leaf keeps its id as the left child
    d.leaf_is_right[nr] = 1;
    d.ls[leaf] = P.lsL;
    d.ls[nr] = P.lsR;
    d.best[leaf] = d_split_none();
    d.best_feature[leaf] = -1;
    d.best[nr] = d_split_none();
    d.best_feature[nr] = -1;
    d.raw[d.raw_len] = 0;
  }
  if (P.la_clear >= 0) d.la_raw[(size_t)P.la_clear * (d.raw_len + 2) + d.raw_len] = 0;
  if (P.kill0 >= 0) d.best[P.kill0].gain = kNegInf;
  if (P.kill1 >= 0) d.best[P.kill1].gain = kNegInf;
  if (P.slot_leaf0 >= 0) d.slot_of_leaf[P.slot_leaf0] = P.slot_val0;
  if (P.slot_leaf1 >= 0) d.slot_of_leaf[P.slot_leaf1] = P.slot_val1;
}

// The control step alone: applies the tree's last split.
__global__ void k_prepare(GrowDev d, int s) {
  if (threadIdx.x != 0) return;
  Prep P;
  if (d.xranks > 1) {
    if (!x_wait<true>(d) || !la_wait<true>(d, s)) atomicOr(&d.ctrl->error, kErrSpinTimeout);
    prep_compute<true>(d, s, P);
  } else {
    prep_compute<false>(d, s, P);
  }
  if (d.has_cat)
    prep_commit<true>(d, P);
  else
    prep_commit<false>(d, P);
  *d.ctrl = P.c;
}

// ------------------------------------------------------------------------------------
// Decode + FixHistogram + compaction + subtraction + scans, one CTA per feature.
// The last CTA to finish does the argmax (scan_leaf_histogram's cross-feature
// argmax, learner.rs:3314-3340, then arg_max over leaves, learner.rs:4537-4551).
// ------------------------------------------------------------------------------------

// Lexicographic order behind the reference's sequential first-max scans: gain
// descending, then feature ascending with -1 last (split_gt, split_info.rs:28-36),
// then position ascending (the scan keeps the first of equal candidates).
__device__ __forceinline__ bool cand_better(double ga, int32_t fa, int32_t ia, double gb,
                                            int32_t fb, int32_t ib) {
  if (ga != gb) return ga > gb;
  const int32_t x = fa == -1 ? 0x7fffffff : fa;
  const int32_t y = fb == -1 ? 0x7fffffff : fb;
  if (x != y) return x < y;
  return ia < ib;
}

struct Cand {
  double g;
  int32_t f, i;
};

__device__ __forceinline__ bool cand_lt(const Cand& a, const Cand& b) {  // a ranks first
  return cand_better(a.g, a.f, a.i, b.g, b.f, b.i);
}

// The first two candidates in pick order. An empty place holds {-inf, -1, INT_MAX},
// which every leaf's candidate outranks (its index is smaller).
struct Cand2 {
  Cand a, b;
};

__device__ __forceinline__ Cand cand_none() { return Cand{kNegInf, -1, 0x7fffffff}; }

__device__ __forceinline__ void cand2_insert(Cand2& t, const Cand& x) {
  if (cand_lt(x, t.a)) {
    t.b = t.a;
    t.a = x;
  } else if (cand_lt(x, t.b)) {
    t.b = x;
  }
}

// Orderable key of a gain (a larger gain has a larger key; -0.0 counts as +0.0). Gains
// are never NaN; key 0 is no candidate.
__device__ __forceinline__ unsigned long long gain_key(double g) {
  const long long b = __double_as_longlong(g == 0.0 ? 0.0 : g);
  return b >= 0 ? (unsigned long long)b ^ 0x8000000000000000ull : ~(unsigned long long)b;
}

__device__ __forceinline__ double key_gain(unsigned long long k) {
  return __longlong_as_double((long long)((k >> 63) ? (k ^ 0x8000000000000000ull) : ~k));
}

// The warp's best feature under split_gt (the larger gain, then the lower feature), from
// each lane's own best {g, f, f} (f = -1: none); every lane gets it. The same order as
// cand_better over the lanes, from two warp max-reductions of the gain key's halves and a
// min-reduction of the tied features.
__device__ __forceinline__ Cand warp_best_feature(const Cand& c) {
  const unsigned long long k = c.f >= 0 ? gain_key(c.g) : 0ull;
  const unsigned hi = (unsigned)(k >> 32), lo = (unsigned)k;
  const unsigned m1 = __reduce_max_sync(0xffffffffu, hi);
  const unsigned m2 = __reduce_max_sync(0xffffffffu, hi == m1 ? lo : 0u);
  const bool tie = k != 0ull && hi == m1 && lo == m2;
  const unsigned fm = __reduce_min_sync(0xffffffffu, tie ? (unsigned)c.f : 0xffffffffu);
  if (fm == 0xffffffffu) return Cand{kNegInf, -1, -1};
  return Cand{key_gain(((unsigned long long)m1 << 32) | m2), (int32_t)fm, (int32_t)fm};
}

// DevSplitInfo as 8-byte words, and word w of d_split_none(): threshold 0 and
// default_left 1 in word 0, gain -inf in word 2, zeros elsewhere.
constexpr int kSplitWords = (int)(sizeof(DevSplitInfo) / 8);
static_assert(offsetof(DevSplitInfo, default_left) == 4 && offsetof(DevSplitInfo, gain) == 16,
              "d_split_none's words");
__device__ __forceinline__ unsigned long long split_none_word(int w) {
  return w == 0 ? (1ull << 32) : w == 2 ? (unsigned long long)__double_as_longlong(kNegInf) : 0ull;
}

__device__ __forceinline__ Cand shfl_cand(const Cand& c, int o) {
  Cand x;
  x.g = __shfl_xor_sync(0xffffffffu, c.g, o);
  x.f = __shfl_xor_sync(0xffffffffu, c.f, o);
  x.i = __shfl_xor_sync(0xffffffffu, c.i, o);
  return x;
}

__device__ __forceinline__ void warp_top2(Cand2& t) {
  for (int o = 16; o > 0; o >>= 1) {
    const Cand xa = shfl_cand(t.a, o), xb = shfl_cand(t.b, o);
    // merge of two ordered pairs (every lane ends with the same pair: a strict order)
    Cand2 m;
    if (cand_lt(xa, t.a)) {
      m.a = xa;
      m.b = cand_lt(t.a, xb) ? t.a : xb;
    } else {
      m.a = t.a;
      m.b = cand_lt(xa, t.b) ? xa : t.b;
    }
    t = m;
  }
}

// Best two splits among the leaves a control step leaves alone: the arg_max inputs of
// learner.rs:4537-4551 other than the leaves being scanned (the two children of the
// applied split, or the root), by one warp. Their best splits are final before the
// step starts, so this runs concurrently with the control step itself. The second is
// the look-ahead's candidate when the first wins the pick.
__device__ Cand2 other_leaves_best(const GrowDev& d) {
  constexpr int kPer = 8;  // leaves per lane: at most 256 leaves
  const GrowCtrl* c = d.ctrl;
  const int lane = threadIdx.x & 31;
  // every read is issued before any is used: one round trip
  double g[kPer];
  int32_t bf[kPer];
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int i = lane + 32 * k;
    g[k] = kNegInf;
    bf[k] = -1;
    if (i < d.L) {
      g[k] = __ldcg(&d.best[i].gain);
      bf[k] = __ldcg(&d.best_feature[i]);
    }
  }
  const int32_t pending = __ldcg(&c->pending);
  const int32_t split_leaf = __ldcg(&c->split_leaf);
  const int32_t num_leaves = __ldcg(&c->num_leaves);
  int32_t ex0 = 0, ex1 = -1;
  if (pending) {
    ex0 = split_leaf;
    ex1 = num_leaves;
  }
  Cand2 t{cand_none(), cand_none()};
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int i = lane + 32 * k;
    if (i < d.L && i != ex0 && i != ex1) cand2_insert(t, Cand{g[k], bf[k], i});
  }
  warp_top2(t);
  return t;
}

// Outcome of the pick at the end of a control step.
struct PickOut {
  DevSplitInfo si[2];  // best split of the smaller / larger scanned leaf
  int32_t bf[2];       // its feature (-1: none)
  int32_t done;        // no leaf has a positive gain: the tree is finished
  int32_t xerr;        // a sliced pick's wait for the other ranks ran out
  int32_t leaf, feature, build_left;
  DevSplitInfo split;  // the split to apply next
  uint32_t si_cat[2][kCatWords];  // left bins of si[] when their feature is categorical
  uint32_t split_cat[kCatWords];  // left bins of `split`
  // the runner-up of the pick (the look-ahead's leaf), valid when la_leaf >= 0
  int32_t la_leaf, la_feature, la_build_left;
  DevSplitInfo la_split;
  uint32_t la_cat[kCatWords];
};

// Cross-feature argmax of both scanned leaves (learner.rs:3314-3321) and the arg_max
// over all leaves (learner.rs:4537-4551, first max under split_gt, learner.rs:1503-1505
// stop rule), by one warp: the feature candidates are reduced with shuffles only.
// Shared memory of a control step besides the per-feature scratch.
// The launch parameters the pick reads, copied into shared memory at the start of the
// control step: the pick is not inlined, and a reference to the launch's GrowDev would copy
// all of it to every thread's stack.
struct PickEnv {
  const DevSplitInfo* scan_out;
  const uint32_t* scan_cat;
  GrowCtrl* ctrl;
  unsigned long long* pick_local;
  unsigned long long* const* peer_pick;
  unsigned long long* pick_flags;
  unsigned long long* const* peer_pick_flags;
  unsigned long long* pick_seq;
  long long xwait_ns;
  int32_t F, slice_begin, slice_end, sliced, lookahead, xrank, xranks;
};

__device__ __forceinline__ void pick_env_set(PickEnv& e, const GrowDev& d) {
  e.scan_out = d.scan_out;
  e.scan_cat = d.scan_cat;
  e.ctrl = d.ctrl;
  e.pick_local = d.pick_local;
  e.peer_pick = d.peer_pick;
  e.pick_flags = d.pick_flags;
  e.peer_pick_flags = d.peer_pick_flags;
  e.pick_seq = d.pick_seq;
  e.xwait_ns = d.xwait_ns;
  e.F = d.F;
  e.slice_begin = d.slice_begin;
  e.slice_end = d.slice_end;
  e.sliced = d.sliced;
  e.lookahead = d.lookahead;
  e.xrank = d.xrank;
  e.xranks = d.xranks;
}

// The pick's inputs besides the scan results (the step's shared state).
struct PickIn {
  Cand2 other;     // the best two leaves the step leaves alone
  Cand wbest[2];   // the features' argmax of a wide slice (wide = 1)
  int32_t live, S, Lg, ok0, ok1, wide;
};

struct CtlSmem {
  Prep prep;
  Cand2 other;                    // the best two leaves the step leaves alone
  DevSplitInfo orec[2];           // ... their best splits (read at the kernel start)
  uint32_t ocat[2][kCatWords];    // ... and their left bins
  int32_t la_prev;                // the previous step's look-ahead leaf (-1: none)
  int32_t oslot[2];               // the other leaves' best two: their histogram slots
  DevFeature ft0;                 // the CTA's first feature
  uint32_t err;                   // the control block's error bits, read by the last CTA
  uint8_t ok[2];                  // the scanned leaves' scan flags
  PickOut pick;
  PickOut pick_dry[3];            // the placeholder runs' outputs (warm_pick)
  PickIn pin[4];                  // the pick's inputs: the real one, the placeholders'
  PickEnv env[3];                 // the launch parameters the pick reads, per placeholder warp
  bool last;
  int32_t wide;                   // the features' argmax was taken by the whole CTA ...
  Cand wbest[2];                  // ... into these (smaller / larger scanned leaf)
  Cand wpart[32][2];              // per-warp partials of that argmax
};

// Slices wider than this take the features' argmax with every thread of the last CTA
// (their gain loads issued together) instead of one warp.
constexpr int kWidePick = 128;

// Best feature of each scanned leaf over this rank's slice, by every thread of the CTA:
// the gains of both leaves (scan_out[0..F), scan_out[F..2F)), strided over the threads and
// loaded kUnroll at a time, reduced in split_gt order (higher gain, then lower feature: a
// strict order, so any partition of the features gives the one-warp loop's result).
template <int CT>
__device__ void block_best_features(const GrowDev& d, int32_t Lg, CtlSmem& cs) {
  constexpr int kUnroll = 4;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  Cand f0{kNegInf, -1, -1}, f1{kNegInf, -1, -1};
  for (int base = d.slice_begin + tid; base < d.slice_end; base += CT * kUnroll) {
    double g0[kUnroll], g1[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int f = base + u * CT;
      g0[u] = f < d.slice_end ? __ldcg(&d.scan_out[f].gain) : kNegInf;
      g1[u] = (f < d.slice_end && Lg >= 0) ? __ldcg(&d.scan_out[d.F + f].gain) : kNegInf;
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int f = base + u * CT;
      if (g0[u] > kNegInf && cand_better(g0[u], f, f, f0.g, f0.f, f0.i)) f0 = Cand{g0[u], f, f};
      if (g1[u] > kNegInf && cand_better(g1[u], f, f, f1.g, f1.f, f1.i)) f1 = Cand{g1[u], f, f};
    }
  }
  f0 = warp_best_feature(f0);
  f1 = warp_best_feature(f1);
  if (lane == 0) {
    cs.wpart[warp][0] = f0;
    cs.wpart[warp][1] = f1;
  }
  __syncthreads();
  if (warp == 0) {
    Cand a{kNegInf, -1, -1}, b{kNegInf, -1, -1};
    if (lane < CT / 32) {
      a = cs.wpart[lane][0];
      b = cs.wpart[lane][1];
    }
    a = warp_best_feature(a);
    b = warp_best_feature(b);
    if (lane == 0) {
      cs.wbest[0] = a;
      cs.wbest[1] = b;
    }
  }
}

// STAGED: `so` / `sc` are the scan results and bin sets in shared memory; otherwise the
// global scan_out / scan_cat. `cs` holds the other leaves' best two and their splits.
template <typename T, bool STAGED>
__device__ __forceinline__ T pick_rd(const T* p) {
  if (STAGED) return *p;
  return __ldcg(p);
}

// The sliced pick's exchange, by the last CTA's warp 0 on every rank. f0 / f1 are this
// rank's best feature of the smaller / larger scanned leaf over its slice (in split_gt
// order, ties to the lower feature); on return they are the best over all ranks, and
// o.si / o.bf / o.si_cat hold those features' splits. Lane q writes this rank's record
// into rank q's pick area (slot [seq parity][this rank]) and releases rank q's flag for
// this rank; lane 0 then waits (bounded) for every rank's flag, and lane q reads rank q's
// record from the local area. A fast rank cannot overwrite a slot that a slow rank still
// reads: it would first have to pass the next step's wait, which needs the slow rank's
// next record.
template <bool CAT, bool STAGED>
__device__ void sliced_pick_exchange(const PickEnv& d, int32_t Lg, const DevSplitInfo* so,
                                     const uint32_t* sc, PickOut& o, Cand& f0, Cand& f1) {
  const int lane = threadIdx.x & 31;
  const unsigned long long target = *reinterpret_cast<const volatile unsigned long long*>(d.pick_seq) + 1;
  const size_t par = (size_t)(target & 1ull);
  // this rank's record, assembled in o by lanes 0 and 1
  if (lane < 2) {
    const Cand& c = lane == 0 ? f0 : f1;
    const bool have = c.f >= 0 && (lane == 0 || Lg >= 0);
    o.si[lane] = have ? so[(size_t)lane * d.F + c.f] : d_split_none();
    o.bf[lane] = have ? c.f : -1;
    if (CAT)
      for (int k = 0; k < kCatWords; ++k)
        o.si_cat[lane][k] = have ? sc[((size_t)lane * d.F + c.f) * kCatWords + k] : 0u;
  }
  __syncwarp();
  if (lane < d.xranks) {
    XPick rec;
    rec.si[0] = o.si[0];
    rec.si[1] = o.si[1];
    rec.bf[0] = o.bf[0];
    rec.bf[1] = o.bf[1];
    for (int k = 0; k < kCatWords; ++k) {
      rec.cat[0][k] = CAT ? o.si_cat[0][k] : 0u;
      rec.cat[1][k] = CAT ? o.si_cat[1][k] : 0u;
    }
    const unsigned long long* src = reinterpret_cast<const unsigned long long*>(&rec);
    unsigned long long* dst =
        d.peer_pick[lane] + (par * kMaxXRanks + (size_t)d.xrank) * kXPickWords;
    for (int k = 0; k < (int)(sizeof(XPick) / 8); ++k) dst[k] = src[k];
    __threadfence_system();
    unsigned long long* flag = d.peer_pick_flags[lane] + d.xrank;
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(flag), "l"(target) : "memory");
  }
  int ok = 1;
  if (lane == 0)
    ok = x_wait_target(&d.ctrl->error, d.xranks, d.pick_flags, target, d.xwait_ns) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  __syncwarp();
  Cand r0{kNegInf, -1, -1}, r1{kNegInf, -1, -1};
  if (ok && lane < d.xranks) {
    const long long* rec = reinterpret_cast<const long long*>(
        d.pick_local + (par * kMaxXRanks + (size_t)lane) * kXPickWords);
    const long long w0 = ld_relaxed_sys(rec + (offsetof(XPick, si) + offsetof(DevSplitInfo, gain)) / 8);
    const long long w1 = ld_relaxed_sys(rec + (offsetof(XPick, si) + sizeof(DevSplitInfo) + offsetof(DevSplitInfo, gain)) / 8);
    const long long wf = ld_relaxed_sys(rec + offsetof(XPick, bf) / 8);
    const int32_t q0 = (int32_t)(wf & 0xffffffffll), q1 = (int32_t)(wf >> 32);
    if (q0 >= 0) r0 = Cand{__longlong_as_double(w0), q0, q0};
    if (q1 >= 0) r1 = Cand{__longlong_as_double(w1), q1, q1};
  }
  r0 = warp_best_feature(r0);
  r1 = warp_best_feature(r1);
  f0 = r0;
  f1 = r1;
  // the owners' records of the winners: lane c copies leaf c's split
  if (ok && lane < 2) {
    const Cand& c = lane == 0 ? r0 : r1;
    if (c.f >= 0) {
      int owner = 0;
      for (int q = 0; q < d.xranks; ++q) {
        const long long wf = ld_relaxed_sys(reinterpret_cast<const long long*>(
            d.pick_local + (par * kMaxXRanks + (size_t)q) * kXPickWords) +
            offsetof(XPick, bf) / 8);
        const int32_t qf = lane == 0 ? (int32_t)(wf & 0xffffffffll) : (int32_t)(wf >> 32);
        if (qf == c.f) owner = q;
      }
      const long long* rec = reinterpret_cast<const long long*>(
          d.pick_local + (par * kMaxXRanks + (size_t)owner) * kXPickWords);
      long long* dst = reinterpret_cast<long long*>(&o.si[lane]);
      const size_t si0 = offsetof(XPick, si) / 8 + (size_t)lane * (sizeof(DevSplitInfo) / 8);
      for (int k = 0; k < (int)(sizeof(DevSplitInfo) / 8); ++k) dst[k] = ld_relaxed_sys(rec + si0 + k);
      o.bf[lane] = c.f;
      if (CAT) {
        const uint32_t* cr = reinterpret_cast<const uint32_t*>(rec + offsetof(XPick, cat) / 8);
        for (int k = 0; k < kCatWords; ++k)
          o.si_cat[lane][k] = (uint32_t)(ld_relaxed_sys(reinterpret_cast<const long long*>(
                                             cr + (size_t)lane * kCatWords + (k & ~1))) >>
                                         (32 * (k & 1)));
      }
    } else {
      o.si[lane] = d_split_none();
      o.bf[lane] = -1;
      if (CAT)
        for (int k = 0; k < kCatWords; ++k) o.si_cat[lane][k] = 0u;
    }
  }
  if (lane == 0) {
    if (!ok) o.xerr = 1;
    *reinterpret_cast<volatile unsigned long long*>(d.pick_seq) = target;
  }
  __syncwarp();
}

// Parts of the pick: the features' argmax of both scanned leaves; their split records and
// the candidates' order; the chosen leaf and runner-up with their records. A real pick
// runs all three; a placeholder run may run any of them alone (on placeholder values).
constexpr int kPickFeatures = 1, kPickRecords = 2, kPickLeaf = 4, kPickAll = 7;

// dry: a placeholder run (no exchange; the output goes to a scratch record).
template <bool CAT, bool STAGED>
__device__ __forceinline__ void pick_warp(const PickEnv& d, const PickIn& in, const CtlSmem& cs,
                                          const DevSplitInfo* so, const uint32_t* sc,
                                          PickOut& o, bool dry, int parts) {
  const int lane = threadIdx.x & 31;
  const bool find = in.live != 0;
  const int32_t S = in.S, Lg = in.Lg;
  const bool xch = !dry && d.sliced != 0;
  Cand2 top = in.other;
  if (lane == 0) o.xerr = 0;
  if (find) {
    const bool ok0 = in.ok0 != 0;
    const bool ok1 = Lg >= 0 && in.ok1 != 0;
    // a placeholder run of the later parts alone starts from the slice's first feature
    const Cand ph = d.slice_end > d.slice_begin ? Cand{1.0, d.slice_begin, d.slice_begin}
                                                : Cand{kNegInf, -1, -1};
    Cand f0 = ph, f1 = ph;
    if (!(parts & kPickFeatures)) {
    } else if (in.wide) {  // taken by the whole CTA (block_best_features)
      f0 = in.wbest[0];
      f1 = in.wbest[1];
    } else {
      f0 = f1 = Cand{kNegInf, -1, -1};
      for (int f = d.slice_begin + lane; f < d.slice_end; f += 32) {
        const double g0 = pick_rd<double, STAGED>(&so[f].gain);
        const double g1 = Lg >= 0 ? pick_rd<double, STAGED>(&so[d.F + f].gain) : kNegInf;
        if (g0 > kNegInf && cand_better(g0, f, f, f0.g, f0.f, f0.i)) f0 = Cand{g0, f, f};
        if (g1 > kNegInf && cand_better(g1, f, f, f1.g, f1.f, f1.i)) f1 = Cand{g1, f, f};
      }
      f0 = warp_best_feature(f0);
      f1 = warp_best_feature(f1);
    }
    if (parts & kPickRecords) {
    if (xch) sliced_pick_exchange<CAT, STAGED>(d, Lg, so, sc, o, f0, f1);
    const int32_t bf0 = ok0 ? f0.f : -1;
    const int32_t bf1 = ok1 ? f1.f : -1;
    if (xch) {
      // the exchange left every rank's best of both leaves in o: apply the scan flags
      if (lane == 0 && bf0 < 0) {
        o.si[0] = d_split_none();
        o.bf[0] = -1;
        if (CAT)
          for (int k = 0; k < kCatWords; ++k) o.si_cat[0][k] = 0u;
      } else if (lane == 1 && bf1 < 0) {
        o.si[1] = d_split_none();
        o.bf[1] = -1;
        if (CAT)
          for (int k = 0; k < kCatWords; ++k) o.si_cat[1][k] = 0u;
      }
    } else {
      // each scanned leaf's best split, one 8-byte word per lane: lanes 0-8 the smaller
      // leaf's, lanes 16-24 the larger leaf's (and their bin sets)
      const int side = lane >> 4, w = lane & 15;
      const int32_t bf = side ? bf1 : bf0;
      const size_t row = (size_t)(side ? d.F : 0) + (size_t)(bf >= 0 ? bf : 0);
      if (w < kSplitWords)
        reinterpret_cast<unsigned long long*>(&o.si[side])[w] =
            bf >= 0 ? pick_rd<unsigned long long, STAGED>(
                          reinterpret_cast<const unsigned long long*>(so + row) + w)
                    : split_none_word(w);
      if (w == 0) o.bf[side] = bf;
      if (CAT && w < kCatWords)
        o.si_cat[side][w] = bf >= 0 ? pick_rd<uint32_t, STAGED>(sc + row * kCatWords + w) : 0u;
    }
    cand2_insert(top, Cand{ok0 ? f0.g : kNegInf, ok0 ? f0.f : -1, S});
    if (Lg >= 0) cand2_insert(top, Cand{ok1 ? f1.g : kNegInf, ok1 ? f1.f : -1, Lg});
    }
  }
  __syncwarp();
  if (!(parts & kPickLeaf)) return;
  // the pick and its runner-up, the same in every lane; their splits are copied one word
  // per lane (lanes 0-8 the pick's, lanes 16-24 the runner-up's)
  const Cand best = top.a;
  const int32_t bl = best.i;
  const bool done = best.g <= 0.0 || bl == 0x7fffffff;
  if (lane == 0) {
    o.la_leaf = -1;
    o.done = done ? 1 : 0;
  }
  if (done) return;
  // an old leaf that wins or runs up is one of the other leaves' best two
  const int sel = (find && bl == S) ? 0 : (find && bl == Lg) ? 1 : -1;
  const int oi = bl == in.other.a.i ? 0 : 1;
  const DevSplitInfo* sp = sel == 0 ? &o.si[0] : sel == 1 ? &o.si[1] : &cs.orec[oi];
  // the runner-up: the next pick chooses it unless a child of this split outranks it
  const Cand ru = top.b;
  const bool la = d.lookahead && ru.i != 0x7fffffff && ru.g > 0.0;
  const int32_t rl = ru.i;
  const int rs = (find && rl == S) ? 0 : (find && rl == Lg) ? 1 : -1;
  const int ri = rl == in.other.a.i ? 0 : 1;
  const DevSplitInfo* rp = rs == 0 ? &o.si[0] : rs == 1 ? &o.si[1] : &cs.orec[ri];
  const int side = lane >> 4, w = lane & 15;
  if (side == 0 || la) {
    if (w < kSplitWords)
      reinterpret_cast<unsigned long long*>(side ? &o.la_split : &o.split)[w] =
          reinterpret_cast<const unsigned long long*>(side ? rp : sp)[w];
    if (CAT && w < kCatWords) {
      if (side == 0)
        o.split_cat[w] = sel >= 0 ? o.si_cat[sel][w] : cs.ocat[oi][w];
      else
        o.la_cat[w] = rs >= 0 ? o.si_cat[rs][w] : cs.ocat[ri][w];
    }
  }
  if (lane == 0) {
    o.leaf = bl;
    o.feature = best.f;
    // accumulate the side the scan expects to be smaller (any side is exact)
    o.build_left = sp->left_count <= sp->right_count ? 1 : 0;
    if (la) {
      o.la_leaf = rl;
      o.la_feature = ru.f;
      o.la_build_left = rp->left_count <= rp->right_count ? 1 : 0;
    }
  }
}

// The pick from staged (shared-memory) or global scan results. Not inlined: its one copy
// of the code is the one the placeholder runs bring into the SM's instruction cache.
template <bool CAT>
__device__ __noinline__ void pick_call(const PickEnv& d, const PickIn& in, const CtlSmem& cs,
                                       bool staged, const DevSplitInfo* so, const uint32_t* sc,
                                       PickOut& o, bool dry, int parts) {
  if (staged)
    pick_warp<CAT, true>(d, in, cs, so, sc, o, dry, parts);
  else
    pick_warp<CAT, false>(d, in, cs, d.scan_out, d.scan_cat, o, dry, parts);
}

// ------------------------------------------------------------------------------------
// Categorical split finder for one leaf by one 256-thread group
// (find_best_threshold_categorical, lgbm-treelearner/src/feature_histogram_categorical.rs
// :96-490, LightGBM FindBestThresholdCategoricalInner). One-hot (num_bin <=
// max_cat_to_onehot): every category is a candidate on its own, one per thread.
// Many-vs-many: the categories with enough rows are ranked by grad / (hess +
// cat_smooth) (a stable sort: ties keep bin order), then two lanes run the reference's
// sequential prefix chains from both ends. `out->bits` gets the bins sent left.
// ------------------------------------------------------------------------------------

struct CatOut {
  DevSplitInfo si;
  uint32_t bits[kCatWords];
};

__device__ void cat_scan(const double* hist, const DevFeature& ft, const DevGainConfig& cfg,
                         const ScanLeaf& leaf, ScanScratch& s, int bar_id, CatOut* out) {
  const int gt = threadIdx.x & (kScanGroup - 1);
  const int lane = gt & 31, wg = gt >> 5;
  const double eps = k_eps();
  const int nb = ft.num_bin, offset = ft.offset;
  const double sum_g = leaf.sum_g;
  const double sum_h = leaf.sum_h + 2.0 * eps;  // bumped at the call site (learner.rs:3104-3109)
  const int32_t nd = leaf.num_data;
  const double cf = (double)nd / sum_h;
  const int bin_start = 1 - offset, bin_end = nb - offset;
  const int nscan = max(bin_end - bin_start, 0);
  const bool onehot = nb <= cfg.max_cat_to_onehot;
  const int32_t min_data = cfg.min_data_in_leaf;
  const double min_hess = cfg.min_sum_hessian_in_leaf;
  const double po = leaf.parent_output;
  // gain_shift uses the original l2 and, without smoothing, no smoothing at all
  double gain_shift;
  if (cfg.use_smoothing) {
    const double sg = cfg.use_l1 ? d_threshold_l1(sum_g, cfg.lambda_l1) : sum_g;
    gain_shift = -fma(2.0 * sg, po, (sum_h + cfg.lambda_l2) * po * po);
  } else {
    DevGainConfig c0 = cfg;
    c0.use_smoothing = 0;
    c0.use_full = cfg.max_delta_step > 0.0 ? 1 : 0;
    gain_shift = d_leaf_gain_full(c0, sum_g, sum_h, nd, 0.0);
  }
  const double mgs = gain_shift + cfg.min_gain_to_split;
  DevGainConfig c2 = cfg;  // per-category gains and outputs: many-vs-many adds cat_l2
  if (!onehot) c2.lambda_l2 = cfg.lambda_l2 + cfg.cat_l2;
  auto gains = [&](double lg, double lh, double rg, double rh, int32_t lc, int32_t rc) {
    return d_leaf_gain_full(c2, lg, lh, lc, po) + d_leaf_gain_full(c2, rg, rh, rc, po);
  };
  double best_gain = kNegInf, best_slg = 0.0, best_slh = 0.0;
  int32_t best_lc = 0, best_thr = -1, best_dir = 1;
  bool splittable = false;
  int32_t* sorted = reinterpret_cast<int32_t*>(s.ph);
  int used = 0;
  if (onehot) {
    const int t = bin_start + gt;
    double cg = kNegInf;
    if (gt < nscan) {
      const double gr = hist[2 * t], he = hist[2 * t + 1];
      const int32_t cnt = d_round_int(he * cf);
      const int32_t other = nd - cnt;
      const double soh = sum_h - he - eps;
      if (!(cnt < min_data || he < min_hess) && other >= min_data && soh >= min_hess) {
        const double v = gains(sum_g - gr, soh, gr, he + eps, other, cnt);
        if (v > mgs) cg = v;
      }
    }
    // first maximum in bin order
    int32_t bt = cg > kNegInf ? t : 0x7fffffff;
    for (int o = 16; o > 0; o >>= 1) {
      const double og = __shfl_xor_sync(0xffffffffu, cg, o);
      const int32_t ot = __shfl_xor_sync(0xffffffffu, bt, o);
      if (og > cg || (og == cg && ot < bt)) {
        cg = og;
        bt = ot;
      }
    }
    if (lane == 0) {
      s.wgain[wg] = cg;
      s.wk[wg] = bt;
    }
    group_sync(bar_id);
    if (gt == 0) {
      for (int w = 1; w < kScanGroup / 32; ++w)
        if (s.wgain[w] > cg || (s.wgain[w] == cg && s.wk[w] < bt)) {
          cg = s.wgain[w];
          bt = s.wk[w];
        }
      if (cg > kNegInf) {
        splittable = true;
        best_gain = cg;
        best_thr = bt;
        best_slg = hist[2 * bt];
        best_slh = hist[2 * bt + 1] + eps;
        best_lc = d_round_int(hist[2 * bt + 1] * cf);
      }
    }
  } else {
    const int t = bin_start + gt;
    bool keep = false;
    double ctr = 0.0;
    if (gt < nscan) {
      keep = (double)d_round_int(hist[2 * t + 1] * cf) >= cfg.cat_smooth;
      ctr = hist[2 * t] / (hist[2 * t + 1] + cfg.cat_smooth);
    }
    // The reference's stable sort by ctr (sort_by with partial_cmp, unordered as Equal; an
    // insertion sort on up to 20 elements): a category moves left past every neighbour with
    // a strictly greater ctr. A NaN ctr (0/0: cat_smooth 0 and a category without rows in
    // this leaf) is ordered with nothing, so it keeps its place among the kept categories
    // and the runs on either side of it are sorted apart. As one total order: key (run,
    // ctr, bin), where a category's run counts the NaNs kept before it and a NaN category
    // opens the run after its own (ctr -inf, first in that run); the bin breaks ties in
    // kept order. A bitonic sort of the 256 keys by the group, 36 compare-exchange stages.
    const bool nan_me = keep && isnan(ctr);
    const unsigned lt = (1u << lane) - 1u;
    const unsigned kb = __ballot_sync(0xffffffffu, keep);
    const unsigned nb = __ballot_sync(0xffffffffu, nan_me);
    if (lane == 0) {
      s.wsum[wg] = __popc(kb);
      s.wpre[wg] = __popc(nb);
    }
    group_sync(bar_id);
    int nan_before = __popc(nb & lt);
    used = 0;
#pragma unroll
    for (int w = 0; w < kScanGroup / 32; ++w) {
      used += s.wsum[w];
      if (w < wg) nan_before += s.wpre[w];
    }
    const int run = nan_me ? nan_before + 1 : nan_before;
    s.pg[gt] = nan_me ? kNegInf : ctr;
    s.pc[gt] = keep ? (run << 9) | t : 0x7ffffe00 | gt;  // left out: last
    group_sync(bar_id);
    for (int k = 2; k <= kScanGroup; k <<= 1) {
      for (int jj = k >> 1; jj > 0; jj >>= 1) {
        const int o = gt ^ jj;
        if (o > gt) {
          const int32_t ka = s.pc[gt], kbb = s.pc[o];
          const double ca = s.pg[gt], cb = s.pg[o];
          const int ra = ka >> 9, rb = kbb >> 9;
          // a after b: a higher run, or the same run and a higher ctr, or equal ctr and a
          // later bin
          const bool after = ra != rb ? ra > rb : (ca != cb ? ca > cb : (ka & 511) > (kbb & 511));
          if (after == ((gt & k) == 0)) {
            s.pc[gt] = kbb;
            s.pc[o] = ka;
            s.pg[gt] = cb;
            s.pg[o] = ca;
          }
        }
        group_sync(bar_id);
      }
    }
    if (gt < used) sorted[gt] = s.pc[gt] & 511;
    group_sync(bar_id);
    if (gt == 0 || gt == 32) {
      const int di = gt == 0 ? 0 : 1;
      const int dir = di == 0 ? 1 : -1;
      int pos = di == 0 ? 0 : used - 1;
      const int max_num_cat = min(cfg.max_cat_threshold, (used + 1) / 2);
      int32_t cnt_group = 0, lc = 0;
      double slg = 0.0, slh = eps;
      double bg = kNegInf, bslg = 0.0, bslh = 0.0;
      int32_t blc = 0, bi = -1, has = 0;
      for (int i = 0; i < used && i < max_num_cat; ++i) {
        const int tt = sorted[pos];
        pos += dir;
        const double gr = hist[2 * tt], he = hist[2 * tt + 1];
        const int32_t cnt = d_round_int(he * cf);
        slg += gr;
        slh += he;
        lc += cnt;
        cnt_group += cnt;
        if (lc < min_data || slh < min_hess) continue;
        const int32_t rc = nd - lc;
        if (rc < min_data || rc < cfg.min_data_per_group) break;
        const double srh = sum_h - slh;
        if (srh < min_hess) break;
        if (cnt_group < cfg.min_data_per_group) continue;
        cnt_group = 0;
        const double v = gains(slg, slh, sum_g - slg, srh, lc, rc);
        if (v <= mgs) continue;
        has = 1;
        if (v > bg) {
          blc = lc;
          bslg = slg;
          bslh = slh;
          bi = i;
          bg = v;
        }
      }
      s.wgain[4 * di + 0] = bg;
      s.wgain[4 * di + 1] = bslg;
      s.wgain[4 * di + 2] = bslh;
      s.wk[4 * di + 0] = blc;
      s.wk[4 * di + 1] = bi;
      s.whas[4 * di] = has;
    }
    group_sync(bar_id);
    if (gt == 0) {
      for (int di = 0; di < 2; ++di) {
        if (s.whas[4 * di]) splittable = true;
        if (s.wk[4 * di + 1] >= 0 && s.wgain[4 * di] > best_gain) {
          best_gain = s.wgain[4 * di];
          best_slg = s.wgain[4 * di + 1];
          best_slh = s.wgain[4 * di + 2];
          best_lc = s.wk[4 * di];
          best_thr = s.wk[4 * di + 1];
          best_dir = di == 0 ? 1 : -1;
        }
      }
    }
  }
  if (gt != 0) return;
  for (int k = 0; k < kCatWords; ++k) out->bits[k] = 0u;
  DevSplitInfo si = d_split_none();
  si.default_left = 0;
  if (splittable && best_thr >= 0) {
    const int32_t rc = nd - best_lc;
    si.threshold = 0;
    si.gain = best_gain - mgs;
    si.left_count = best_lc;
    si.right_count = rc;
    si.left_output = d_leaf_output_full(c2, c2.use_smoothing, best_slg, best_slh, best_lc, po);
    si.left_sum_gradient = best_slg;
    si.left_sum_hessian = best_slh - eps;
    si.right_output = d_leaf_output_full(c2, c2.use_smoothing, sum_g - best_slg,
                                         sum_h - best_slh, rc, po);
    si.right_sum_gradient = sum_g - best_slg;
    si.right_sum_hessian = sum_h - best_slh - eps;
    if (onehot) {
      const int b = best_thr + offset;
      out->bits[b >> 5] |= 1u << (b & 31);
    } else {
      for (int i = 0; i <= best_thr; ++i) {
        const int b = (best_dir == 1 ? sorted[i] : sorted[used - 1 - i]) + offset;
        out->bits[b >> 5] |= 1u << (b & 31);
      }
    }
  }
  out->si = si;
}

// Shared memory of one feature's control-step work (decode, FixHistogram, scans).
struct FixScanSmem {
  double hist[2][2 * kMaxBins];
  ScanScratch scan[4];
  ScanCand cand[4];
  double fix[2 * kMaxBins / 32][3];  // per-warp exact sums for FixHistogram
  CatOut cat[2];                     // categorical results of the two scanned leaves
};

// Feature f of one control step (every thread of the CTA calls it): the smaller child's
// histogram cells (accumulated by the partition, or derived from the parent), FixHistogram,
// compaction, the larger child by subtraction, and the REVERSE/FORWARD scans of both
// children.
template <bool CAT, bool PEER, int CT>
__device__ void fixscan_feature(const GrowDev& d, const Prep& P, int f, const DevFeature& ft,
                                FixScanSmem& sm, int s) {
  static_assert(CT == 1024 || (CT == 256 && !CAT), "control-step CTA sizes");
  const int tid = threadIdx.x;
  const int nb = ft.num_bin;
  // one histogram cell per thread (2*num_bin <= 512 cells)
  const bool mine = tid < 2 * nb;
  const size_t cell = 2 * (size_t)ft.bin_off + tid;
  // Every global read of this feature's cells is issued here, before any store or branch
  // on loaded data, so their round trips overlap: the accumulated child (its left or
  // right rows, all devices summed; per-tile partials are integers, summed in any order),
  // the parent's integer cells and the larger child's parent slot.
  const int32_t S = P.S, Lg = P.Lg;
  long long bv = 0, pv = 0;
  double parent = 0.0;
  const int nt = P.priv_tiles;
  const int as = P.acc_slot;
  if (mine) {
    if (nt == 0) bv = as >= 0 ? la_sum<PEER>(d, as, cell) : raw_sum<PEER>(d, cell);
    if (P.live && P.applied) pv = __ldcg(d.rawpool + (size_t)P.leaf * d.raw_len + cell);
    if (P.live && Lg >= 0) parent = d.pool[(size_t)P.lslot * d.slot_len + ft.slot_off + tid];
  }
  const bool used_f =
      !P.live || !P.use_sub || d.splittable[(size_t)P.mask_leaf * d.F + f] != 0;
  // Per-tile partials: the two halves of the CTA load tiles [0, 8) and [8, 16) of their
  // cell, all in one round trip (integers: any order of summation).
  long long tsum = 0;
  if (nt > 0) {
    const int half = tid / (CT / 2), c2 = tid % (CT / 2);
    const size_t rl = (size_t)d.raw_len;
    const long long* pp =
        (as >= 0 ? d.la_partials + (size_t)as * d.private_tiles * rl : d.partials) +
        2 * (size_t)ft.bin_off + c2 + (size_t)(half * kHalfTiles) * rl;
    const int nh = c2 < 2 * nb ? min(nt - half * kHalfTiles, kHalfTiles) : 0;
    long long a[kHalfTiles];
#pragma unroll
    for (int j = 0; j < kHalfTiles; ++j) a[j] = j < nh ? __ldcg(pp + (size_t)j * rl) : 0ll;
#pragma unroll
    for (int j = 1; j < kHalfTiles; ++j) a[0] += a[j];
    tsum = a[0];
  }
  if (nt > kHalfTiles) {  // uniform: the upper half hands its sums to the lower half
    long long* xs = reinterpret_cast<long long*>(sm.hist[1]);
    if (tid >= CT / 2) xs[tid - CT / 2] = tsum;
    __syncthreads();
    if (tid < CT / 2) tsum += xs[tid];
  }
  if (mine && nt > 0) bv = tsum;
  // clear the accumulator for the next partition (on one device a look-ahead hit left it
  // untouched; with several, `raw` is the other exchange buffer, read by every rank at the
  // previous step), and this step's look-ahead slot for its next look-ahead kernel
  if (mine && P.priv_tiles == 0 && (PEER || P.acc_slot < 0)) d.raw[cell] = 0;
  if (mine && P.la_clear >= 0) d.la_raw[(size_t)P.la_clear * (d.raw_len + 2) + cell] = 0;
  if (P.live) {
    const bool used = used_f;
    if (used) {
      const DevGhParams& p = *d.ghp;
      const DevLeafSplits lss = P.lsS;
      const bool buildable = leaf_buildable(lss);
      double v = 0.0;
      if (mine) {
        // Integer histograms of both children: the accumulated side as is, the other as
        // parent - accumulated. Exact, so the smaller child's cells equal a direct build.
        long long sv = bv;
        if (P.applied) {
          long long* pr = d.rawpool + (size_t)P.leaf * d.raw_len + cell;
          const long long ov = pv - bv;
          const bool bl = P.c.build_left != 0;
          const long long lv = bl ? bv : ov;
          const long long rv = bl ? ov : bv;
          *pr = lv;
          d.rawpool[(size_t)P.nr * d.raw_len + cell] = rv;
          sv = P.smaller_is_left ? lv : rv;
        } else {
          d.rawpool[cell] = bv;  // root
        }
        if (buildable) v = (tid & 1) ? decode_h(p, sv) : decode_g(p, sv);
        sm.hist[0][tid] = v;
      }
      __syncthreads();
      ctl_mark(d, s, CP_LOADED);
      // FixHistogram (fix_histogram.rs:50-81): the most-frequent-bin cell becomes the leaf
      // sum minus the other cells, subtracted in ascending order. With quantized
      // gradients every cell is an exact multiple of one unit u. When every partial
      // result of that chain is representable (checked below from exact sums) each
      // subtraction is exact, so the chain equals sum - (other cells summed in any
      // order). Otherwise the sequential chain runs.
      const int mfb = ft.most_freq_bin;
      if (buildable && mfb > 0 && mfb < nb) {
        const int w = tid == 0 ? 0 : 1;
        bool fast = false;
        double fixed = 0.0;
        if (p.mode != GH_FLOAT) {
          double xg = 0.0, xh = 0.0, ag = 0.0;
          if (mine && (tid >> 1) != mfb) {
            if (tid & 1) {
              xh = sm.hist[0][tid];
            } else {
              xg = sm.hist[0][tid];
              ag = fabs(xg);
            }
          }
          // exact in any order: partial sums are multiples of u below 2^53 u (checked)
          for (int o = 16; o > 0; o >>= 1) {
            xg += __shfl_xor_sync(0xffffffffu, xg, o);
            xh += __shfl_xor_sync(0xffffffffu, xh, o);
            ag += __shfl_xor_sync(0xffffffffu, ag, o);
          }
          if ((tid & 31) == 0 && tid < 2 * kMaxBins) {
            sm.fix[tid >> 5][0] = xg;
            sm.fix[tid >> 5][1] = xh;
            sm.fix[tid >> 5][2] = ag;
          }
          __syncthreads();
          if (tid == 0 || tid == 32) {
            const int nw = (2 * nb + 31) >> 5;
            double cs = 0.0, as = 0.0;
            for (int k = 0; k < nw; ++k) {
              cs += sm.fix[k][w];
              as += sm.fix[k][2];
            }
            const double unit = w == 0 ? p.unit_g : p.unit_h;
            double u = unit;
            if (p.mode == GH_QPACK) {  // the f32 level's ulp divides every level
              int e = 0;
              frexp(unit, &e);
              u = ldexp(1.0, e - 24);
            }
            const double sum = w == 0 ? lss.sum_g : lss.sum_h;
            const double lim = ldexp(u, 52);
            if (unit > 0.0) {
              if (w == 0) {
                const double m = sum / u;  // power-of-two division: exact
                fast = m == trunc(m) && fabs(sum) + as < lim;
              } else {
                fast = sum >= 0.0 && cs <= 2.0 * sum && sum < lim;
              }
            }
            fixed = sum - cs;
          }
        }
        if ((tid == 0 || tid == 32)) {
          if (!fast) {
            double acc = w == 0 ? lss.sum_g : lss.sum_h;
            const double* hv = &sm.hist[0][w];
            acc = seq_sub(hv, 2, mfb, acc);
            acc = seq_sub(hv + 2 * (mfb + 1), 2, nb - mfb - 1, acc);
            fixed = acc;
          }
          sm.hist[0][2 * mfb + w] = fixed;
        }
      }
      __syncthreads();
      // compact_histogram (learner.rs:4460-4486)
      double sv = mine ? sm.hist[0][tid] : 0.0;
      if (ft.offset > 0) {
        const int src = tid + 2 * ft.offset;
        sv = (mine && src < 2 * nb) ? sm.hist[0][src] : 0.0;
        __syncthreads();
        if (mine) sm.hist[0][tid] = sv;
      }
      // store the smaller child's slot; larger = parent - smaller in the parent's slot
      if (mine) {
        d.pool[(size_t)P.sslot * d.slot_len + ft.slot_off + tid] = sv;
        if (Lg >= 0) {
          const double lv = parent - sv;
          d.pool[(size_t)P.lslot * d.slot_len + ft.slot_off + tid] = lv;
          sm.hist[1][tid] = lv;
        }
      }
      __syncthreads();
      ctl_mark(d, s, CP_FIXED);
      const int grp = tid / (CT / 4);  // (leaf, direction) group
      const int sel = grp >> 1;
      const bool fwd = (grp & 1) != 0;
      const int32_t leaf = sel == 0 ? S : Lg;
      const bool is_cat = CAT && (ft.flags & kFeatCategorical) != 0;
      if (leaf >= 0) {
        const DevLeafSplits ls = sel == 0 ? P.lsS : P.lsLg;
        if (leaf_buildable(ls)) {
          ScanLeaf sl{ls.sum_g, ls.sum_h, ls.weight, ls.num_data};
          if (!is_cat)
            scan_direction<CT / 4>(sm.hist[sel], ft, d.gain, sl, fwd, sm.scan[grp], 1 + grp,
                                   &sm.cand[grp]);
          else if (!fwd)  // bin_type dispatch (learner.rs:3099-3149)
            cat_scan(sm.hist[sel], ft, d.gain, sl, sm.scan[grp], 1 + grp, &sm.cat[sel]);
        }
      }
      __syncthreads();
      ctl_mark(d, s, CP_SCANNED);
      if (tid == 0 || tid == 32) {
        const int sl_i = tid == 0 ? 0 : 1;
        const int32_t leaf2 = sl_i == 0 ? S : Lg;
        if (leaf2 >= 0) {
          const DevLeafSplits ls = sl_i == 0 ? P.lsS : P.lsLg;
          const bool scannable = leaf_buildable(ls);
          if (f == d.slice_begin) d.scan_ok[sl_i] = scannable ? 1 : 0;
          DevSplitInfo si = d_split_none();
          if (scannable) {
            if (is_cat) {
              si = sm.cat[sl_i].si;
              uint32_t* dst = d.scan_cat + ((size_t)sl_i * d.F + f) * kCatWords;
              for (int k = 0; k < kCatWords; ++k) dst[k] = sm.cat[sl_i].bits[k];
            } else {
              ScanLeaf sl{ls.sum_g, ls.sum_h, ls.weight, ls.num_data};
              si = finalize_split(d.gain, sl, sm.cand[2 * sl_i], sm.cand[2 * sl_i + 1]);
            }
          }
          d.scan_out[sl_i * d.F + f] = si;
          // the scanned leaf's children may split this feature only if it has a split
          // (learner.rs:2003-2020)
          if (scannable) d.splittable[(size_t)leaf2 * d.F + f] = si.gain > kNegInf ? 1 : 0;
        }
      }
    } else if (tid == 0) {
      d.scan_out[f] = d_split_none();
      d.scan_out[d.F + f] = d_split_none();
      if (leaf_buildable(P.lsS)) d.splittable[(size_t)S * d.F + f] = 0;
      if (Lg >= 0 && leaf_buildable(P.lsLg)) d.splittable[(size_t)Lg * d.F + f] = 0;
      if (f == d.slice_begin) {
        d.scan_ok[0] = leaf_buildable(P.lsS) ? 1 : 0;
        d.scan_ok[1] = Lg >= 0 && leaf_buildable(P.lsLg) ? 1 : 0;
      }
    }
  }
}


// The last CTA copies every feature's scan result of both leaves (and their bin sets)
// into the per-feature scratch in one round trip when they fit there.
constexpr int kStageFeatures =
    (int)(sizeof(FixScanSmem) / (2 * (sizeof(DevSplitInfo) + kCatWords * sizeof(uint32_t))));
static_assert(sizeof(DevSplitInfo) % 8 == 0, "scan results are copied as 8-byte words");

// One control step by the CTAs [0, min(F, gridDim.x)), each taking features
// blockIdx.x, blockIdx.x + gridDim.x, ...: apply the pending split, scan the two leaves,
// and -- in the CTA that finishes last -- pick the next split and write the control block.
// nctl: the control CTAs (the launch's first nctl CTAs). main_part: run by every control CTA
// after the prep when the pending split still needs its main partition (the fused control
// step partitions it itself, then redoes the prep; elsewhere a no-op, the partition having
// run as its own launch).
template <bool CAT, bool PEER, int CT, class MainPart>
__device__ void control_step(const GrowDev& d, int s, FixScanSmem& sm, CtlSmem& cs, int nctl,
                             MainPart&& main_part) {
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int fb = d.slice_begin, fe = d.slice_end;  // this rank's features
  const int nparts = min(fe - fb, nctl);
  if (tid == 0) {
    if (!x_la_wait<PEER>(d, s)) atomicOr(&d.ctrl->error, kErrSpinTimeout);
    prep_compute<PEER>(d, s, cs.prep);
  } else if (warp == 1) {
    // the best two of the leaves this step leaves alone (final before the step starts;
    // the last CTA reads their splits with its other inputs)
    const Cand2 o = other_leaves_best(d);
    if ((tid & 31) == 0) cs.other = o;
  } else if (tid == 64) {
    if (fb + (int)blockIdx.x < fe) cs.ft0 = d.feat[fb + blockIdx.x];
  } else {
    // Placeholder warps k = 0, 1, 2 (warps 4, 8, 12 with 1024 threads, on warp 0's
    // scheduler partition; warps 4, 5, 6 with 256): each copies the pick's launch
    // parameters, and with warm_pick runs part k of the pick on placeholder inputs (two
    // old leaves with positive gains, both scanned leaves live) into its own scratch
    // record. A run takes the real pick's path through that part of the code, so that the
    // code is in the SM's instruction cache when the last CTA runs the pick; it reads only
    // shared memory or in-range scan results. The three parts run side by side, each
    // shorter than the prep above.
    const int k = CT == 1024 ? (warp - 4) >> 2 : warp - 4;
    const bool ph_warp = warp >= 4 && k < 3 && (CT != 1024 || (warp & 3) == 0);
    if (ph_warp) {
      const bool st = d.F <= kStageFeatures;
      if ((tid & 31) == 0) {
        pick_env_set(cs.env[k], d);
        PickIn& in = cs.pin[1 + k];
        in.other.a = Cand{1e300, 0, 0x7ffffffe};
        in.other.b = Cand{1e299, 0, 0x7ffffffd};
        in.wbest[0] = in.wbest[1] = Cand{kNegInf, -1, -1};
        in.live = 1;
        in.S = 0x7ffffffc;
        in.Lg = 0x7ffffffb;
        in.ok0 = in.ok1 = 1;
        in.wide = !st && (fe - fb) > kWidePick ? 1 : 0;
      }
      __syncwarp();
      if (d.warm_pick) {
        const DevSplitInfo* so = reinterpret_cast<const DevSplitInfo*>(&sm);
        const uint32_t* sc = reinterpret_cast<const uint32_t*>(so + 2 * kStageFeatures);
        pick_call<CAT>(cs.env[k], cs.pin[1 + k], cs, st, so, sc, cs.pick_dry[k], true, 1 << k);
      }
    }
  }
  __syncthreads();
  ctl_mark(d, s, CP_PREP);
  if (cs.prep.main_needed) main_part();
  if (PEER && d.sliced) {
    // With feature slices the owners of all features sum every rank's buffers, so this
    // rank clears every cell of its next accumulator and of the look-ahead slot it
    // releases (fixscan_feature clears only its slice's): the CTAs share the cells. Both
    // were last read at the previous step, which every rank has finished.
    const Prep& P = cs.prep;
    const int64_t rl = d.raw_len;
    const int64_t per = (rl + nctl - 1) / nctl;
    const int64_t lo = per * blockIdx.x, hi = min(rl, lo + per);
    long long* la = P.la_clear >= 0 ? d.la_raw + (size_t)P.la_clear * (rl + 2) : nullptr;
    for (int64_t i = lo + tid; i < hi; i += CT) {
      d.raw[i] = 0;
      if (la) la[i] = 0;
    }
  }
  for (int f = fb + blockIdx.x; f < fe; f += nctl) {
    // the CTA's first feature was read while the pending split was applied
    const DevFeature ft = f == fb + (int)blockIdx.x ? cs.ft0 : d.feat[f];
    fixscan_feature<CAT, PEER, CT>(d, cs.prep, f, ft, sm, s);
    __syncthreads();
  }
  ctl_mark(d, s, CP_FEATURES);
  // Arrival: the barrier orders every thread's writes before thread 0's release, and the
  // CTA that arrives last acquires all of them (acq_rel add) before its barrier.
  __syncthreads();
  if (tid == 0) {
    const uint32_t t = atom_add_acq_rel_gpu(&d.ctrl->scan_counter, 1u);
    cs.last = (t == (uint32_t)nparts - 1);
  }
  __syncthreads();
  if (!cs.last) return;
  const Prep& P = cs.prep;
  // One round trip for everything the pick reads that other CTAs wrote: the scan results
  // (into the per-feature scratch, when they fit), the scan flags and the error bits.
  const bool staged = d.F <= kStageFeatures;
  DevSplitInfo* so = reinterpret_cast<DevSplitInfo*>(&sm);
  uint32_t* sc = reinterpret_cast<uint32_t*>(so + 2 * kStageFeatures);
  if (staged) {
    const int nw = d.F * (int)(2 * sizeof(DevSplitInfo) / 8);
    const unsigned long long* src = reinterpret_cast<const unsigned long long*>(d.scan_out);
    unsigned long long* dst = reinterpret_cast<unsigned long long*>(so);
    for (int i = tid; i < nw; i += CT) dst[i] = __ldcg(src + i);
    if (CAT)
      for (int i = tid; i < 2 * d.F * kCatWords; i += CT) sc[i] = __ldcg(d.scan_cat + i);
  }
  if (tid == CT - 32) {
    cs.ok[0] = __ldcg(&d.scan_ok[0]);
    cs.ok[1] = __ldcg(&d.scan_ok[1]);
    cs.err = *reinterpret_cast<volatile uint32_t*>(&d.ctrl->error);  // other CTAs' bits
  } else if (warp == 2) {
    // the other leaves' best two: their splits, bin sets and histogram slots; and the
    // previous step's look-ahead leaf
    const int lane = tid & 31;
    if (lane < 2) {
      const int32_t i = lane == 0 ? cs.other.a.i : cs.other.b.i;
      if (i != 0x7fffffff) {
        cs.orec[lane] = d.best[i];
        if (CAT)
          for (int k = 0; k < kCatWords; ++k)
            cs.ocat[lane][k] = d.best_cat[(size_t)i * kCatWords + k];
      }
    } else if (lane == 4 || lane == 5) {
      const int32_t i = lane == 4 ? cs.other.a.i : cs.other.b.i;
      cs.oslot[lane - 4] = i != 0x7fffffff ? d.slot_of_leaf[i] : -1;
    } else if (lane == 2) {
      int32_t lp = -1;
      if (d.lookahead && s >= 1) {
        const LookAhead& q = d.la[(s - 1) & (kLaSlots - 1)];
        if (q.active) lp = q.leaf;
      }
      cs.la_prev = lp;
    }
  }
  if (warp == 1 && (tid & 31) == 0) prep_commit<CAT>(d, P);
  // wide slices: the features' argmax by the whole CTA (its gain loads issued together)
  const bool wide = !staged && P.live && !P.c.done && (fe - fb) > kWidePick;
  if (tid == 0) cs.wide = wide ? 1 : 0;
  if (wide) block_best_features<CT>(d, P.Lg, cs);
  __syncthreads();
  ctl_mark(d, s, CP_STAGED);
  if (warp == 0 && !P.c.done) {
    if ((tid & 31) == 0)
      cs.pin[0] = PickIn{cs.other, {cs.wbest[0], cs.wbest[1]}, P.live, P.S, P.Lg, cs.ok[0],
                         cs.ok[1], cs.wide};
    __syncwarp();
    pick_call<CAT>(cs.env[0], cs.pin[0], cs, staged, so, sc, cs.pick, false, kPickAll);
  }
  __syncthreads();
  ctl_mark(d, s, CP_PICKED);
  // The next step reads the chosen leaf's integer and f64 histogram rows, which the
  // partitions' streaming has usually pushed out of L2 since the leaf was scanned: bring
  // them back now, one bulk prefetch per 16 KB.
  // Rows above kPrefetchMax bytes (wide data) are left out: one SM's bulk prefetches of
  // megabytes hold the kernel's end back longer than the next step's many CTAs take to
  // read the rows themselves.
  constexpr uint32_t kPrefetchMax = 512u << 10;
  if (warp == 1 && !P.c.done && !cs.pick.done && (uint64_t)d.raw_len * 8u <= kPrefetchMax) {
    const int32_t b = cs.pick.leaf;
    const int32_t slot = (P.live && b == P.S)    ? P.sslot
                         : (P.live && b == P.Lg) ? P.lslot
                         : cs.oslot[b == cs.other.a.i ? 0 : 1];
    const uint32_t bytes = (uint32_t)d.raw_len * 8u;
    const int lane = tid & 31;
    constexpr uint32_t kChunk = 16384;
    const uint32_t nck = (bytes + kChunk - 1) / kChunk;
    for (uint32_t k = lane; k < 2 * nck; k += 32) {
      const bool pool_row = k >= nck;
      if (pool_row && slot < 0) continue;
      const uint32_t off = (pool_row ? k - nck : k) * kChunk;
      const char* base = pool_row ? reinterpret_cast<const char*>(d.pool + (size_t)slot * d.slot_len)
                                  : reinterpret_cast<const char*>(d.rawpool + (size_t)b * d.raw_len);
      prefetch_l2_bulk(base + off, min(kChunk, bytes - off));
    }
  }
  if (tid == 0) {
    GrowCtrl c = P.c;
    c.scan_counter = 0;
    if (!c.done) {
      if (P.live) {
        d.best[P.S] = cs.pick.si[0];
        d.best_feature[P.S] = cs.pick.bf[0];
        if (CAT)
          for (int k = 0; k < kCatWords; ++k)
            d.best_cat[(size_t)P.S * kCatWords + k] = cs.pick.si_cat[0][k];
        if (P.Lg >= 0) {
          d.best[P.Lg] = cs.pick.si[1];
          d.best_feature[P.Lg] = cs.pick.bf[1];
          if (CAT)
            for (int k = 0; k < kCatWords; ++k)
              d.best_cat[(size_t)P.Lg * kCatWords + k] = cs.pick.si_cat[1][k];
        }
      }
      if (cs.pick.done) {
        c.done = 1;
      } else {
        c.pending = 1;
        c.split_leaf = cs.pick.leaf;
        c.split_feature = cs.pick.feature;
        c.split = cs.pick.split;
        c.build_left = cs.pick.build_left;
        if (CAT)
          for (int k = 0; k < kCatWords; ++k) d.split_cat[k] = cs.pick.split_cat[k];
        // the previous step's look-ahead partitioned this leaf already (it may still be
        // running; the step that applies the split waits for it)
        if (d.lookahead && s >= 1 && cs.la_prev == cs.pick.leaf)
          c.pend_la = 1 + ((s - 1) & (kLaSlots - 1));
      }
    }
    // The previous step's look-ahead is of no use when this pick took another leaf (or
    // ended the tree): its kernel, which may still be partitioning a big leaf beside this
    // step, stops taking tiles and leaves the SMs to the main partition. Its slot is never
    // read; it is cleared as every unused slot is.
    if (d.la_cancel && d.lookahead && s >= 1 && cs.la_prev >= 0 &&
        !(!c.done && c.pend_la == 1 + ((s - 1) & (kLaSlots - 1))))
      d.la[(s - 1) & (kLaSlots - 1)].cancel = 1;
    c.error |= cs.err;
    if (!P.c.done && cs.pick.xerr) c.error |= kErrSpinTimeout;
    if (c.error & kErrSpinTimeout) c.done = 1;  // a rank stopped answering: end the tree
    // this step's look-ahead: the runner-up of the pick (its kernel runs next to the
    // following control step; slot s % 2 was consumed and cleared above)
    if (d.lookahead && s <= d.L - 3) {
      LookAhead r{};
      r.epoch = c.epoch;
      if (!c.done && c.pending && cs.pick.la_leaf >= 0) {
        r.active = 1;
        r.leaf = cs.pick.la_leaf;
        r.feature = cs.pick.la_feature;
        r.build = s < d.L - 3 ? 1 : 0;  // the last look-ahead feeds no scan
        r.build_left = cs.pick.la_build_left;
        r.split = cs.pick.la_split;
        if (CAT)
          for (int k = 0; k < kCatWords; ++k) r.cat[k] = cs.pick.la_cat[k];
      }
      d.la[s & (kLaSlots - 1)] = r;
    }
    if (d.mainrec) {
      // the next (fused) control step's main partition: the split it partitions when the
      // look-ahead did not, with the epoch this control block carries and fresh counters
      LookAhead m{};
      m.active = (!c.done && c.pending && !c.pend_la) ? 1 : 0;
      if (m.active) {
        m.leaf = c.split_leaf;
        m.feature = c.split_feature;
        m.build = 1;
        m.build_left = c.build_left;
        m.epoch = c.epoch;
        m.split = c.split;
        if (CAT)
          for (int k = 0; k < kCatWords; ++k) m.cat[k] = cs.pick.split_cat[k];
      }
      d.mainrec[(s + 1) & 1] = m;
    }
    *d.ctrl = c;
  }
  ctl_mark(d, s, CP_WRITTEN);
}

template <bool CAT, bool PEER, int CT>
__global__ void __launch_bounds__(CT, CT == 1024 ? 1 : 4) k_fixscan(GrowDev d, int s) {
  const SpanStamp span(d);
  __shared__ FixScanSmem sm;
  __shared__ CtlSmem cs;
  control_step<CAT, PEER, CT>(d, s, sm, cs, (int)gridDim.x, [] {});
}

// ------------------------------------------------------------------------------------
// Stable partition of one leaf's rows, single pass with decoupled look-back.
// Left rows keep ascending position order from the front of the leaf's range;
// right rows are written from the back (a stable reversal), so no second pass
// over the data is needed to learn the left total.
// ------------------------------------------------------------------------------------

__device__ __forceinline__ unsigned long long pack_status(uint32_t epoch, uint32_t flag,
                                                          uint32_t v) {
  return ((unsigned long long)(epoch & 0xffffffu) << 40) | ((unsigned long long)flag << 32) | v;
}

struct PartitionTile {
  // returns false on look-back timeout
  __device__ static bool run(const uint8_t* __restrict__ bins, int32_t stride, bool packed4,
                             const DevFeature& ft, int32_t feature, uint32_t threshold,
                             bool default_left, const uint32_t* __restrict__ src,
                             bool identity, uint32_t* __restrict__ dst, int32_t begin,
                             int32_t count, int32_t tile, uint32_t epoch,
                             unsigned long long* status, int32_t* left_total,
                             const uint32_t* cat = nullptr) {
    __shared__ int32_t s_warp[kPartThreads / 32];
    __shared__ int32_t s_prefix;
    __shared__ int32_t s_ok;
    const int tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const int32_t base = tile * kPartTile;
    uint32_t rows[kPartItems];
    uint32_t leftmask = 0, validmask = 0;
#pragma unroll
    for (int j = 0; j < kPartItems; ++j) {
      const int32_t p = base + tid * kPartItems + j;
      if (p < count) {
        const uint32_t row = identity ? (uint32_t)(begin + p) : src[begin + p];
        rows[j] = row;
        const int32_t bin = (int32_t)row_bin(bins + (size_t)row * stride, feature, packed4);
        validmask |= 1u << j;
        const bool gr = cat ? d_cat_go_right(cat, bin)
                            : ((ft.flags & kFeatMissingRoute)
                                   ? !d_route_left_missing(ft, threshold, default_left, bin)
                                   : d_go_right(ft, threshold, default_left, bin));
        if (!gr) leftmask |= 1u << j;
      }
    }
    const int32_t my_left = __popc(leftmask);
    int32_t incl = my_left;
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += n;
    }
    if (lane == 31) s_warp[warp] = incl;
    __syncthreads();
    int32_t warp_off = 0, tile_left = 0;
    for (int w = 0; w < kPartThreads / 32; ++w) {
      const int32_t v = s_warp[w];
      if (w < warp) warp_off += v;
      tile_left += v;
    }
    const int32_t excl = warp_off + incl - my_left;
    if (warp == 0) {
      // Decoupled look-back, one warp reading a window of 32 predecessor words per step.
      // Flag 1 = tile aggregate, 2 = inclusive prefix; a word of another epoch is "not
      // ready". Positions before tile 0 read as an inclusive prefix of 0.
      int32_t prefix = 0;
      int32_t ok = 1;
      if (lane == 0) {
        __threadfence();
        atomicExch(&status[tile], pack_status(epoch, tile == 0 ? 2u : 1u, (uint32_t)tile_left));
      }
      if (tile > 0) {
        const uint32_t ep = epoch & 0xffffffu;
        int32_t j_end = tile;
        long long spins = 0;
        while (true) {
          const int32_t j = j_end - 32 + lane;
          uint32_t fl = 2u, val = 0u;
          if (j >= 0) {
            const unsigned long long w =
                *reinterpret_cast<volatile unsigned long long*>(&status[j]);
            fl = ((uint32_t)(w >> 40) == ep) ? ((uint32_t)(w >> 32) & 0xffu) : 0u;
            val = (uint32_t)(w & 0xffffffffull);
          }
          const uint32_t pref = __ballot_sync(0xffffffffu, fl == 2u);
          const uint32_t notready = __ballot_sync(0xffffffffu, fl == 0u);
          const int hp = pref ? 31 - __clz(pref) : -1;  // nearest inclusive prefix
          const uint32_t need = hp >= 0 ? (0xffffffffu << hp) : 0xffffffffu;
          if (notready & need) {
            if (++spins > kSpinLimit) {
              ok = 0;
              break;
            }
            __nanosleep(20);
            continue;
          }
          int32_t v = (lane >= hp) ? (int32_t)val : 0;
          for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
          prefix += v;
          if (hp >= 0) break;
          j_end -= 32;
        }
        if (lane == 0 && ok) {
          __threadfence();
          atomicExch(&status[tile], pack_status(epoch, 2u, (uint32_t)(prefix + tile_left)));
        }
      }
      if (lane == 0) {
        atomicAdd(left_total, tile_left);
        s_prefix = prefix;
        s_ok = ok;
      }
    }
    __syncthreads();
    const int32_t prefix_left = s_prefix;
    const bool ok = s_ok != 0;
    if (ok) {
      const int32_t prefix_right = base - prefix_left;
      int32_t lrank = excl;
      const int32_t my_base = tid * kPartItems;
#pragma unroll
      for (int j = 0; j < kPartItems; ++j) {
        if (!((validmask >> j) & 1u)) continue;
        if ((leftmask >> j) & 1u) {
          dst[begin + prefix_left + lrank] = rows[j];
          ++lrank;
        } else {
          const int32_t rrank = (my_base + j) - lrank;  // rights before this item in tile
          dst[begin + count - 1 - (prefix_right + rrank)] = rows[j];
        }
      }
    }
    __syncthreads();
    return ok;
  }
};

__global__ void __launch_bounds__(kPartThreads) k_partition(GrowDev d) {
  const SpanStamp span(d);
  __shared__ int32_t s_tile;
  GrowCtrl* c = d.ctrl;
  if (c->done || !c->pending) return;
  const int32_t leaf = c->split_leaf;
  const int32_t f = c->split_feature;
  const DevFeature ft = d.feat[f];
  const int32_t begin = d.leaf_begin[leaf];
  const int32_t count = d.leaf_count[leaf];
  const int32_t src = d.leaf_buf[leaf];
  const uint32_t* sp = src == 1 ? d.idx1 : d.idx0;
  uint32_t* dp = src == 1 ? d.idx0 : d.idx1;
  const int32_t ntiles = (count + kPartTile - 1) / kPartTile;
  if (blockIdx.x == 0 && threadIdx.x == 0) c->rows_parted += count;
  const uint32_t epoch = c->epoch;
  const uint32_t thr = c->split.threshold;
  const bool dl = c->split.default_left != 0;
  while (true) {
    if (threadIdx.x == 0) s_tile = (int32_t)atomicAdd(&c->part_ticket, 1u);
    __syncthreads();
    const int32_t tile = s_tile;
    __syncthreads();
    if (tile >= ntiles) break;
    const bool ok = PartitionTile::run(d.bins, d.stride, d.packed4 != 0, ft, f, thr, dl, sp,
                                       src == 2, dp, begin,
                                       count, tile, epoch, d.part_status, &c->part_left_total,
                                       (ft.flags & kFeatCategorical) ? d.split_cat : nullptr);
    if (!ok) {
      if (threadIdx.x == 0) {
        atomicOr(&c->error, kErrSpinTimeout);
        c->done = 1;
      }
      break;
    }
  }
}

// ------------------------------------------------------------------------------------
// Partition fused with the histogram build of one child (quantized, <= 4 quant bins,
// every feature in one shared-memory group). The partition already fetches each row's
// 32-byte bin sector to route it; the rows that go to the accumulated side
// (GrowCtrl::build_left) are added to the CTA's shared histogram straight from those
// registers, while warp 0 waits on the look-back. The other child's histogram is
// derived exactly in k_fixscan as parent - accumulated. One CTA of 1024 threads per
// SM; tiles are the standalone partition's 2048-row tiles (same status words).
// ------------------------------------------------------------------------------------

constexpr int kFpThreads = 1024;
constexpr int kFpItems = 2;
static_assert(kFpThreads * kFpItems == kPartTile, "fused tiles are partition tiles");
constexpr int kFpMaxChunks = 2;  // 16-feature row chunks held in registers per item

// A status word carries its flag and count together in one aligned 64-bit store, and
// readers use nothing else that the writer stored before it: a relaxed store suffices
// (no fence, no read-modify-write round trip on the critical path).
__device__ __forceinline__ void publish_status(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Decoupled look-back of one tile by warp 0 (status words as in PartitionTile).
// Returns the exclusive prefix of left rows; *ok = 0 after kSpinLimit polls.
__device__ __forceinline__ int32_t tile_lookback(unsigned long long* status, int32_t tile,
                                                 uint32_t epoch, int32_t tile_left,
                                                 int32_t* ok) {
  const int lane = threadIdx.x & 31;
  int32_t prefix = 0;
  *ok = 1;
  if (lane == 0)
    publish_status(&status[tile], pack_status(epoch, tile == 0 ? 2u : 1u, (uint32_t)tile_left));
  if (tile == 0) return 0;
  const uint32_t ep = epoch & 0xffffffu;
  int32_t j_end = tile;
  long long spins = 0;
  while (true) {
    const int32_t j = j_end - 32 + lane;
    uint32_t fl = 2u, val = 0u;
    if (j >= 0) {
      const unsigned long long w = *reinterpret_cast<volatile unsigned long long*>(&status[j]);
      fl = ((uint32_t)(w >> 40) == ep) ? ((uint32_t)(w >> 32) & 0xffu) : 0u;
      val = (uint32_t)(w & 0xffffffffull);
    }
    const uint32_t pref = __ballot_sync(0xffffffffu, fl == 2u);
    const uint32_t notready = __ballot_sync(0xffffffffu, fl == 0u);
    const int hp = pref ? 31 - __clz(pref) : -1;
    const uint32_t need = hp >= 0 ? (0xffffffffu << hp) : 0xffffffffu;
    if (notready & need) {
      if (++spins > kSpinLimit) {
        *ok = 0;
        return 0;
      }
      __nanosleep(20);
      continue;
    }
    int32_t v = (lane >= hp) ? (int32_t)val : 0;
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    prefix += v;
    if (hp >= 0) break;
    j_end -= 32;
  }
  if (lane == 0) publish_status(&status[tile], pack_status(epoch, 2u, (uint32_t)(prefix + tile_left)));
  return prefix;
}

// Shared memory of the fused partition besides its accumulators.
struct PartSmem {
  int32_t warp[kFpThreads / 32];
  int32_t tile, prefix, ok;
  int32_t ntiles;  // tiles of the partitioned leaf (set once the leaf is known)
  int32_t nb[128];
  int32_t boff[128];
  uint32_t mask[4];
  uint32_t cat[kCatWords];  // left bins of a categorical split
};

// f32 gradients in the fused partition: the 64-bit fixed-point values of the build
// (GhValue<GH_FLOAT>) added with two native 64-bit shared atomics per (row, feature) into
// g64 / h64, cell = (feature << SHIFT) + bin. The sums are exact integers, so the child
// histogram is the one the separate build kernel would produce.
template <int SHIFT, int NCH, bool MASKED>
__device__ __forceinline__ void f32_row_regs(const uint4 (&w)[NCH], long long a, long long b,
                                             unsigned long long* g64, const uint32_t* mask,
                                             uint32_t tail) {
#pragma unroll
  for (int ch = 0; ch < NCH; ++ch) {
    const uint32_t words[4] = {w[ch].x, w[ch].y, w[ch].z, w[ch].w};
    const uint32_t m16 = MASKED ? ((mask[ch >> 1] >> ((ch & 1) * 16)) & 0xffffu) : tail;
    const bool test = MASKED || ch == NCH - 1;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (test && !((m16 >> j) & 1u)) continue;
      const uint32_t bin = (words[j >> 2] >> (8 * (j & 3))) & 0xffu;
      unsigned long long* cell = g64 + ((16 * ch + j) << SHIFT) + bin;
      atomicAdd(cell, (unsigned long long)a);
      atomicAdd(cell + kQ4MaxCells, (unsigned long long)b);
    }
  }
}

// One fused partition by the whole grid (every thread of every CTA calls it); `sm` holds
// the accumulators. Quantized (F32 false): hot | c3 | cold_g | cold_q, kQ4MaxCells u32
// words each. f32 gradients: g64 | h64, kQ4MaxCells u64 words each (the same bytes).
// mrec (the fused control step's main partition): the split, its status-word epoch, the
// tile tickets and the finished-tile counter come from this record, written by the control
// step before, instead of the control block (which this kernel's own last CTA rewrites);
// the outputs are the main partition's. Each CTA adds the tiles it finished to mrec->done,
// with release semantics, after its histogram is flushed.
template <int SHIFT, int NCH, bool F32, bool PACK4>
__device__ void partition_q4_phase(const GrowDev& d, int build, int la, uint32_t* sm,
                                   PartSmem& ps_, LookAhead* mrec = nullptr) {
  uint32_t* const done_ctr = mrec ? &mrec->done : nullptr;
  static_assert(NCH <= kFpMaxChunks, "row chunks held in registers");
  int32_t* s_warp = ps_.warp;
  int32_t& s_tile = ps_.tile;
  int32_t& s_prefix = ps_.prefix;
  int32_t& s_ok = ps_.ok;
  int32_t* s_nb = ps_.nb;
  int32_t* s_boff = ps_.boff;
  uint32_t* s_mask = ps_.mask;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // la >= 0: the look-ahead partition of slot la (its leaf, split, counters, status
  // words and accumulator); otherwise the pending split of the control block
  LookAhead* const rec = la >= 0 ? d.la + la : nullptr;
  uint32_t* const ticket = rec ? &rec->ticket : mrec ? &mrec->ticket : &d.ctrl->part_ticket;
  const unsigned long long t_entry = d.ctl_phase ? global_ns() : 0ull;
  if (!rec) {
    // The main partition has nothing to do after the tree, or when the look-ahead did this
    // partition (most splits): one read of the control block decides, before any other
    // request, so that such a launch costs a single round trip.
    if (tid == 0) {
      const GrowCtrl* c0 = d.ctrl;
      s_ok = mrec ? (mrec->active ? 1 : 0) : (c0->done || !c0->pending || c0->pend_la) ? 0 : 1;
    }
    __syncthreads();
    if (!s_ok) return;
  }
  // the first tile ticket is taken before anything else is read: its round trip overlaps
  // the reads below (a ticket taken when there is nothing to do is harmless)
  if (tid == 0) s_tile = (int32_t)atomicAdd(ticket, 1u);
  // the dataset's feature table does not depend on the split: read it first
  if (build)
    for (int fl = tid; fl < d.F; fl += kFpThreads) {
      const DevFeature g = d.feat[fl];
      s_nb[fl] = g.num_bin;
      s_boff[fl] = g.bin_off;
    }
  GrowCtrl* c = d.ctrl;
  int32_t leaf, f;
  uint32_t epoch, thr;
  bool dl, build_left;
  const uint32_t* cat_src;
  unsigned long long* status;
  long long* raw;
  long long* partials;
  if (rec) {
    if (!rec->active) return;
    leaf = rec->leaf;
    f = rec->feature;
    epoch = rec->epoch;
    thr = rec->split.threshold;
    dl = rec->split.default_left != 0;
    build_left = rec->build_left != 0;
    if (!rec->build) build = 0;
    cat_src = rec->cat;
    status = d.la_status;
    raw = d.la_raw + (size_t)la * (d.raw_len + 2);
    partials = d.la_partials + (size_t)la * d.private_tiles * d.raw_len;
  } else if (mrec) {
    leaf = mrec->leaf;
    f = mrec->feature;
    epoch = mrec->epoch;
    thr = mrec->split.threshold;
    dl = mrec->split.default_left != 0;
    build_left = mrec->build_left != 0;
    cat_src = mrec->cat;
    status = d.part_status;
    raw = d.raw;
    partials = d.partials;
  } else {
    // nothing to do after the tree, or when the look-ahead did this partition
    if (c->done || !c->pending || c->pend_la) return;
    leaf = c->split_leaf;
    f = c->split_feature;
    epoch = c->epoch;
    thr = c->split.threshold;
    dl = c->split.default_left != 0;
    build_left = c->build_left != 0;
    cat_src = d.split_cat;
    status = d.part_status;
    raw = d.raw;
    partials = d.partials;
  }
  const DevFeature ft = d.feat[f];
  const int32_t begin = d.leaf_begin[leaf];
  const int32_t count = d.leaf_count[leaf];
  const int32_t src = d.leaf_buf[leaf];
  const uint32_t* sp = src == 1 ? d.idx1 : d.idx0;
  uint32_t* dp = src == 1 ? d.idx0 : d.idx1;
  const bool identity = src == 2;
  const int32_t ntiles = (count + kPartTile - 1) / kPartTile;
  if (tid == 0) ps_.ntiles = ntiles;
  const bool is_cat = (ft.flags & kFeatCategorical) != 0;
  const int nf = d.F;
  const int cap = nf << SHIFT;
  // the children keep the features their parent could split (learner.rs:2003-2020); the
  // mask is read with the leaf's range
  if (build && tid < 128) {
    const uint8_t* ps = d.splittable + (size_t)leaf * d.F;
    const uint32_t m = __ballot_sync(0xffffffffu, tid < nf && (d.sliced || ps[tid] != 0));
    if ((tid & 31) == 0) s_mask[tid >> 5] = m;
  }
  // few tiles: every CTA takes exactly one tile and stores its own partial histogram
  // (plain stores, summed by the next control step) instead of adding it atomically
  const bool priv = build && ntiles <= d.private_tiles;
  if (blockIdx.x == 0 && tid == 0) {
    if (rec) {
      rec->ran = 1;
      rec->rows = count;
    } else {
      c->rows_parted += count;
      if (build) c->num_builds += 1;
      if (done_ctr) c->rows_parted_ctl += count;
    }
  }
  if (is_cat && tid < kCatWords) ps_.cat[tid] = cat_src[tid];
  __syncthreads();
  int32_t tile = s_tile;
  if (tile >= ntiles) return;
  const int32_t my_tile = tile;
  part_mark(d, rec != nullptr, PP_START, t_entry);
  uint32_t* hot = sm;
  uint32_t* c3 = sm + kQ4MaxCells;
  int32_t* cold_g = reinterpret_cast<int32_t*>(sm + 2 * kQ4MaxCells);
  int32_t* cold_q = reinterpret_cast<int32_t*>(sm + 3 * kQ4MaxCells);
  unsigned long long* g64 = reinterpret_cast<unsigned long long*>(sm);
  if (build) {
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
    if (F32) {
      uint4* a4 = reinterpret_cast<uint4*>(g64);
      uint4* b4 = reinterpret_cast<uint4*>(g64 + kQ4MaxCells);
      for (int i = tid; i < (cap + 1) / 2; i += kFpThreads) {
        a4[i] = z;
        b4[i] = z;
      }
    } else {
      uint4* h4 = reinterpret_cast<uint4*>(hot);
      uint4* c4 = reinterpret_cast<uint4*>(c3);
      for (int i = tid; i < (cap + 3) / 4; i += kFpThreads) {
        h4[i] = z;
        c4[i] = z;
      }
    }
  }
  __syncthreads();
  if (d.ctl_phase) part_mark(d, rec != nullptr, PP_READY, global_ns());
  Q4Mask qm = q4_mask<NCH>(s_mask, nf);
  const uint16_t* gq = reinterpret_cast<const uint16_t*>(d.gh);
  const float2* gf = reinterpret_cast<const float2*>(d.gh);
  const double scale_g = F32 ? d.ghp->scale_g : 0.0;
  const double scale_h = F32 ? d.ghp->scale_h : 0.0;
  const int fch = f >> 4, fw = (f >> 2) & 3, fsh = (f & 3) * 8;
  const size_t stride = (size_t)d.stride;
  bool folded = false;
  int32_t acc_rows = 0;
  int32_t cta_left = 0;
  long long cta_built = 0;
  bool failed = false;
  bool cancelled = false;
  uint32_t tiles_done = 0;
  while (true) {
    const int32_t base = tile * kPartTile;
    // a look-ahead's cancel flag, read as the tile starts and used before the next ticket
    int32_t cancel_seen = 0;
    if (rec && tid == 0) cancel_seen = *reinterpret_cast<volatile int32_t*>(&rec->cancel);
    uint32_t rows[kFpItems];
    uint4 w[kFpItems][NCH];
    uint16_t q[kFpItems];
    float2 fv[kFpItems];
    uint32_t leftmask = 0, validmask = 0;
#pragma unroll
    for (int j = 0; j < kFpItems; ++j) {
      const int32_t p = base + tid * kFpItems + j;
      rows[j] = 0;
      if (p < count) {
        rows[j] = identity ? (uint32_t)(begin + p) : sp[begin + p];
        validmask |= 1u << j;
      }
    }
#pragma unroll
    for (int j = 0; j < kFpItems; ++j) {
      if ((validmask >> j) & 1u) {
        load_row<NCH, PACK4>(d.bins + (size_t)rows[j] * stride, w[j]);
        if (F32)
          fv[j] = build ? gf[rows[j]] : make_float2(0.0f, 0.0f);
        else
          q[j] = build ? gq[rows[j]] : (uint16_t)0;
      } else {
#pragma unroll
        for (int ch = 0; ch < NCH; ++ch) w[j][ch] = make_uint4(0u, 0u, 0u, 0u);
        q[j] = 0;
        fv[j] = make_float2(0.0f, 0.0f);
      }
    }
#pragma unroll
    for (int j = 0; j < kFpItems; ++j) {
      if (!((validmask >> j) & 1u)) continue;
      uint4 v = w[j][0];
#pragma unroll
      for (int ch = 1; ch < NCH; ++ch)
        if (ch == fch) v = w[j][ch];
      const uint32_t word = fw == 0 ? v.x : fw == 1 ? v.y : fw == 2 ? v.z : v.w;
      const int32_t bin = (int32_t)((word >> fsh) & 0xffu);
      const bool gr = is_cat ? d_cat_go_right(ps_.cat, bin) : d_go_right(ft, thr, dl, bin);
      if (!gr) leftmask |= 1u << j;
    }
    const int32_t my_left = __popc(leftmask);
    int32_t incl = my_left;
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += n;
    }
    if (lane == 31) s_warp[warp] = incl;
    __syncthreads();
    if (d.ctl_phase && tile == my_tile) part_mark(d, rec != nullptr, PP_LOADED, global_ns());
    int32_t warp_off = 0, tile_left = 0;
#pragma unroll 8
    for (int wi = 0; wi < kFpThreads / 32; ++wi) {
      const int32_t v = s_warp[wi];
      if (wi < warp) warp_off += v;
      tile_left += v;
    }
    const int32_t excl = warp_off + incl - my_left;
    if (warp == 0) {
      int32_t ok = 1;
      const int32_t prefix = tile_lookback(status, tile, epoch, tile_left, &ok);
      if (lane == 0) {
        s_prefix = prefix;
        s_ok = ok;
      }
    }
    // accumulate the chosen side while warp 0 looks back
    if (build) {
#pragma unroll
      for (int j = 0; j < kFpItems; ++j) {
        if (!((validmask >> j) & 1u)) continue;
        const bool is_left = (leftmask >> j) & 1u;
        if (is_left != build_left) continue;
        if (F32) {
          const long long a = __double2ll_rn((double)fv[j].x * scale_g);
          const long long b = __double2ll_rn((double)fv[j].y * scale_h);
          if (qm.full)
            f32_row_regs<SHIFT, NCH, false>(w[j], a, b, g64, qm.w, qm.tail);
          else
            f32_row_regs<SHIFT, NCH, true>(w[j], a, b, g64, qm.w, qm.tail);
        } else {
          const int qg = (int)(int8_t)(q[j] & 0xff), qh = (int)(int8_t)(q[j] >> 8);
          if (qm.full)
            q4_row_regs<SHIFT, NCH, false>(w[j], qg + (qh << 16), qh == 3, hot, qm.w, qm.tail);
          else
            q4_row_regs<SHIFT, NCH, true>(w[j], qg + (qh << 16), qh == 3, hot, qm.w, qm.tail);
        }
      }
    }
    __syncthreads();
    if (d.ctl_phase && tile == my_tile) part_mark(d, rec != nullptr, PP_PREFIX, global_ns());
    const int32_t prefix_left = s_prefix;
    if (s_ok == 0) {
      failed = true;
      break;
    }
    {
      const int32_t prefix_right = base - prefix_left;
      int32_t lrank = excl;
      const int32_t my_base = tid * kFpItems;
#pragma unroll
      for (int j = 0; j < kFpItems; ++j) {
        if (!((validmask >> j) & 1u)) continue;
        if ((leftmask >> j) & 1u) {
          dp[begin + prefix_left + lrank] = rows[j];
          ++lrank;
        } else {
          const int32_t rrank = (my_base + j) - lrank;
          dp[begin + count - 1 - (prefix_right + rrank)] = rows[j];
        }
      }
    }
    const int32_t valid = min(kPartTile, count - base);
    const int32_t built = build_left ? tile_left : valid - tile_left;
    cta_left += tile_left;
    cta_built += built;
    acc_rows += built;
    ++tiles_done;
    if (priv) break;
    // A cancelled look-ahead takes no further ticket, so no tile is left untaken behind
    // a ticket that a later tile's look-back would wait on.
    if (tid == 0) s_tile = cancel_seen ? -1 : (int32_t)atomicAdd(ticket, 1u);
    __syncthreads();
    tile = s_tile;
    if (tile < 0) {
      cancelled = true;
      break;
    }
    if (tile >= ntiles) break;
    // fold the 16-bit packed fields before the next tile could overflow them (the 64-bit
    // f32 cells need no fold)
    if (!F32 && build && acc_rows + kPartTile > kQ4Chunk) {
      for (int s2 = tid; s2 < cap; s2 += kFpThreads) {
        const int32_t v = (int32_t)hot[s2];
        const int32_t lo = (int32_t)(int16_t)(v & 0xffff);
        const int32_t hi = (v - lo) >> 16;
        cold_g[s2] = folded ? cold_g[s2] + lo : lo;
        cold_q[s2] = folded ? cold_q[s2] + hi : hi;
        hot[s2] = 0u;
      }
      folded = true;
      acc_rows = 0;
      __syncthreads();
    }
  }
  if (d.ctl_phase) part_mark(d, rec != nullptr, PP_TILES, global_ns());
  if (failed) {
    if (tid == 0) {
      if (rec) {
        rec->failed = 1;  // reported by the control step that consumes the slot
      } else {
        atomicOr(&c->error, kErrSpinTimeout);
        c->done = 1;
      }
    }
    return;
  }
  if (cancelled) return;  // its slot is never read
  if (build) {
    __syncthreads();
    long long* part = partials + (size_t)my_tile * d.raw_len;
    for (int s2 = tid; s2 < cap; s2 += kFpThreads) {
      const int fl = s2 >> SHIFT;
      const int bin = s2 & ((1 << SHIFT) - 1);
      if (fl >= nf || bin >= s_nb[fl]) continue;
      long long g, h;
      if (F32) {
        g = (long long)g64[s2];
        h = (long long)g64[kQ4MaxCells + s2];
      } else {
        const int32_t v = (int32_t)hot[s2];
        const int32_t lo = (int32_t)(int16_t)(v & 0xffff);
        g = (folded ? (long long)cold_g[s2] : 0ll) + lo;
        const long long qsum = (folded ? (long long)cold_q[s2] : 0ll) + ((v - lo) >> 16);
        const long long n3 = (long long)c3[s2];
        h = (qsum - 3 * n3) | (n3 << 32);
      }
      const size_t gb = (size_t)(s_boff[fl] + bin);
      if (priv) {
        *reinterpret_cast<longlong2*>(&part[2 * gb]) = make_longlong2(g, h);
      } else {
        if (g)
          atomicAdd(reinterpret_cast<unsigned long long*>(&raw[2 * gb]), (unsigned long long)g);
        if (h)
          atomicAdd(reinterpret_cast<unsigned long long*>(&raw[2 * gb + 1]),
                    (unsigned long long)h);
      }
    }
  }
  if (tid == 0) {
    atomicAdd(rec ? &rec->left_total : &c->part_left_total, cta_left);
    atomicAdd(reinterpret_cast<unsigned long long*>(&raw[d.raw_len]),
              (unsigned long long)(long long)cta_left);
    if (build)
      atomicAdd(reinterpret_cast<unsigned long long*>(rec ? &rec->built : &c->rows_built),
                (unsigned long long)cta_built);
    if (build && done_ctr)
      atomicAdd(reinterpret_cast<unsigned long long*>(&c->rows_built_ctl),
                (unsigned long long)cta_built);
  }
  if (d.ctl_phase) {  // uniform over the CTA (a launch parameter)
    __syncthreads();
    part_mark(d, rec != nullptr, PP_FLUSHED, global_ns());
  }
  if (done_ctr) {
    // the barrier orders every thread's flush before thread 0's release
    __syncthreads();
    if (tid == 0) atom_add_acq_rel_gpu(done_ctr, tiles_done);
  }
}


template <int SHIFT, int NCH, bool F32, bool PACK4 = false>
__global__ void __launch_bounds__(kFpThreads, 1) k_partition_q4(GrowDev d, int build, int la) {
  const SpanStamp span(d);
  extern __shared__ uint32_t sm[];
  __shared__ PartSmem ps;
  partition_q4_phase<SHIFT, NCH, F32, PACK4>(d, build, la, sm, ps);
  producer_signal(d);
}

// Bounded wait (thread 0) until `want` tiles of the main partition are done, or the tree was
// ended (a look-back that gave up sets done). False when the wait ran out.
__device__ __noinline__ bool wait_part_done(GrowCtrl* c, const uint32_t* done, uint32_t want) {
  // twice the look-back's limit: a partition CTA that gives up ends the tree first
  for (long long spins = 0;; ++spins) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(done) : "memory");
    if (v >= want) return true;
    if (*reinterpret_cast<volatile int32_t*>(&c->done)) return true;
    if (spins > 2 * kSpinLimit) return false;
    __nanosleep(32);
  }
}

// The control step of split step s with the main partition of the split picked at step
// s - 1 folded in: when the previous look-ahead did not partition that leaf, the control
// CTAs (the first nctl) and the helper CTAs after them partition it first (the main
// partition's own code, tiles by ticket), the control CTAs wait for every tile, redo the
// prep and go on. Otherwise the helpers return after one read of their record, and the
// split costs one launch instead of two (control step, then a main partition that finds
// nothing to do). The partition's split, epoch, tickets and tile counter come from
// mainrec[s & 1], which the previous control step wrote: a helper placed on an SM only
// after this kernel's last CTA rewrote the control block still reads its own step's
// record, finds every ticket drawn (or nothing to do) and returns; the next step's record
// is the other one. No CTA waits on a CTA that has not taken a tile: a control CTA
// leaves the tile loop only once every ticket is drawn, by CTAs that are running.
template <int SHIFT, int NCH, bool F32, bool PACK4>
__global__ void __launch_bounds__(1024, 1)
    k_fixscan_part(GrowDev d, int s, GrowDev dp, int nctl) {
  static_assert(kFpThreads == 1024, "the fused control step runs the partition's CTA shape");
  const SpanStamp span(d);
  extern __shared__ uint32_t smp[];
  __shared__ FixScanSmem sm;
  __shared__ CtlSmem cs;
  __shared__ PartSmem ps;
  LookAhead* const mrec = dp.mainrec + (s & 1);
  if ((int)blockIdx.x >= nctl) {
    partition_q4_phase<SHIFT, NCH, F32, PACK4>(dp, 1, -1, smp, ps, mrec);
    return;
  }
  control_step<false, false, 1024>(d, s, sm, cs, nctl, [&] {
    partition_q4_phase<SHIFT, NCH, F32, PACK4>(dp, 1, -1, smp, ps, mrec);
    if (threadIdx.x == 0) {
      if (!wait_part_done(d.ctrl, &mrec->done, (uint32_t)ps.ntiles))
        atomicOr(&d.ctrl->error, kErrSpinTimeout);
      prep_compute<false>(d, s, cs.prep);  // with the partition's counts
    }
    __syncthreads();
  });
}

using FixscanPartKernel = void (*)(GrowDev, int, GrowDev, int);
__host__ FixscanPartKernel fixscan_part_kernel(int shift, int nch, bool f32, bool pack4) {
  if (shift != 8 || pack4) return nullptr;
  if (nch == 1) return f32 ? k_fixscan_part<8, 1, true, false> : k_fixscan_part<8, 1, false, false>;
  if (nch == 2) return f32 ? k_fixscan_part<8, 2, true, false> : k_fixscan_part<8, 2, false, false>;
  return nullptr;
}

using PartQ4Kernel = void (*)(GrowDev, int, int);
__host__ PartQ4Kernel part_q4_kernel(int shift, int nch, bool f32 = false, bool pack4 = false) {
  if (pack4) {  // 4-bit rows (shift 4)
    if (shift == 4 && nch == 1) return f32 ? k_partition_q4<4, 1, true, true> : k_partition_q4<4, 1, false, true>;
    if (shift == 4 && nch == 2) return f32 ? k_partition_q4<4, 2, true, true> : k_partition_q4<4, 2, false, true>;
    return nullptr;
  }
#define PQ4_CASE(S, N) \
  if (shift == S && nch == N) return f32 ? k_partition_q4<S, N, true> : k_partition_q4<S, N, false>;
  PQ4_CASE(4, 1) PQ4_CASE(4, 2) PQ4_CASE(5, 1) PQ4_CASE(5, 2) PQ4_CASE(6, 1) PQ4_CASE(6, 2)
  PQ4_CASE(7, 1) PQ4_CASE(7, 2) PQ4_CASE(8, 1) PQ4_CASE(8, 2)
#undef PQ4_CASE
  return nullptr;
}

// ---------------------------- standalone per-op kernels ----------------------------

__global__ void k_hist_standalone(const uint8_t* bins, int32_t stride, int64_t n,
                                  const float2* gh, int32_t num_bin, double sg, double sh,
                                  long long* raw) {
  __shared__ unsigned long long acc[2 * kMaxBins];
  for (int i = threadIdx.x; i < 2 * num_bin; i += blockDim.x) acc[i] = 0ull;
  __syncthreads();
  for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < n;
       r += (int64_t)gridDim.x * blockDim.x) {
    const float2 v = gh[r];
    const uint32_t bin = bins[(size_t)r * stride];
    atomicAdd(&acc[2 * bin], (unsigned long long)__double2ll_rn((double)v.x * sg));
    atomicAdd(&acc[2 * bin + 1], (unsigned long long)__double2ll_rn((double)v.y * sh));
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 2 * num_bin; i += blockDim.x)
    if (acc[i]) atomicAdd((unsigned long long*)&raw[i], acc[i]);
}

__global__ void __launch_bounds__(512) k_scan_standalone(const double* hist,
                                                         const DevFeature* feats,
                                                         DevGainConfig cfg, DevLeafSplits ls,
                                                         DevSplitInfo* out) {
  __shared__ double s_hist[2 * kMaxBins];
  __shared__ ScanScratch s_scan[2];
  __shared__ ScanCand s_cand[2];
  const DevFeature ft = feats[blockIdx.x];
  for (int i = threadIdx.x; i < 2 * ft.num_bin; i += blockDim.x)
    s_hist[i] = hist[ft.slot_off + i];
  __syncthreads();
  const int grp = threadIdx.x >> 8;
  ScanLeaf sl{ls.sum_g, ls.sum_h, ls.weight, ls.num_data};
  scan_direction<256>(s_hist, ft, cfg, sl, grp == 1, s_scan[grp], 1 + grp, &s_cand[grp]);
  __syncthreads();
  if (threadIdx.x == 0) out[blockIdx.x] = finalize_split(cfg, sl, s_cand[0], s_cand[1]);
}

__global__ void __launch_bounds__(kPartThreads) k_partition_standalone(
    const uint8_t* bins, int32_t stride, int32_t feature, const DevFeature* feat,
    uint32_t threshold, int32_t default_left, int32_t count, uint32_t* dst,
    unsigned long long* status, int32_t* left_total, uint32_t* ticket, uint32_t* error) {
  __shared__ int32_t s_tile;
  const DevFeature ft = *feat;
  const int32_t ntiles = (count + kPartTile - 1) / kPartTile;
  while (true) {
    if (threadIdx.x == 0) s_tile = (int32_t)atomicAdd(ticket, 1u);
    __syncthreads();
    const int32_t tile = s_tile;
    __syncthreads();
    if (tile >= ntiles) break;
    if (!PartitionTile::run(bins, stride, false, ft, feature, threshold, default_left != 0, nullptr,
                            true, dst, 0, count, tile, 1u, status, left_total)) {
      // the look-back gave up: this tile's rows were not written, so the result is void
      if (threadIdx.x == 0) atomicOr(error, kErrSpinTimeout);
      break;
    }
  }
}

__global__ void k_gather_partition(GrowDev d, uint32_t* out) {
  const int leaf = blockIdx.y;
  if (leaf >= d.ctrl->num_leaves) return;
  const int32_t begin = d.leaf_begin[leaf];
  const int32_t count = d.leaf_count[leaf];
  const int32_t buf = d.leaf_buf[leaf];
  const uint32_t* src = buf == 1 ? d.idx1 : d.idx0;
  for (int32_t p = blockIdx.x * blockDim.x + threadIdx.x; p < count; p += gridDim.x * blockDim.x)
    out[begin + p] = buf == 2 ? (uint32_t)(begin + p) : src[begin + p];
}

__global__ void k_subtract(const double* a, const double* b, double* o, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    o[i] = a[i] - b[i];
}

}  // namespace

int build_smem_bytes_per_bin(int gh_mode) { return gh_mode == GH_QPACK ? 8 : 16; }

static int g_num_sms = 0;

static int num_sms() {
  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_num_sms <= 0) g_num_sms = 148;
  }
  return g_num_sms;
}

int LaunchProfiler::begin(cudaStream_t st, int c) {
  if (n >= cap) return -1;
  cls[n] = c;
  cudaEventRecord(ev[n][0], st);
  return n++;
}

void LaunchProfiler::end(cudaStream_t st, int slot) {
  if (slot >= 0) cudaEventRecord(ev[slot][1], st);
}

#define PROF_BEGIN(c) const int _slot = prof ? prof->begin(st, (c)) : -1
#define PROF_END() \
  do {             \
    if (prof) prof->end(st, _slot); \
  } while (0)

// The partition accumulates the child itself for packed quantized gradients and for f32
// gradients, when every feature fits one shared-memory layout (feature << shift) + bin.
bool fused_partition_supported(int gh_mode, int num_features, int shift, int nch, bool pack4) {
  return (gh_mode == GH_QPACK || gh_mode == GH_FLOAT) && num_features <= 128 &&
         (num_features << shift) <= kQ4MaxCells && nch <= kFpMaxChunks &&
         part_q4_kernel(shift, nch, gh_mode == GH_FLOAT, pack4) != nullptr;
}

size_t fused_partition_smem() { return (size_t)4 * sizeof(uint32_t) * kQ4MaxCells; }


// One tree: root build, then per split the control step + scans (k_fixscan) and the
// partition, which in the fused mode also accumulates one child's histogram (else a
// build kernel follows). With several devices the accumulated child (d.raw: raw_len
// integer cells + the left-row count) is summed over them after every build, so every
// device takes the same decisions.
void launch_tree(const GrowDev& d_in, int build_blocks, size_t build_smem, cudaStream_t st,
                 LaunchProfiler* prof, const DeviceComm* comm, const LookAheadStreams* las) {
  const int sms = num_sms();
  // Look-ahead partitions on the second stream (one device, fused partition): the kernel
  // of step s starts after control step s and must end before control step s + 2, which
  // consumes or clears its slot. The kernels see the flag only when they are launched.
  const bool la_on = d_in.lookahead && las && d_in.fused &&
                     (d_in.xranks > 1 ? d_in.la_xbuf != nullptr : !comm);
  GrowDev d = d_in;
  d.lookahead = la_on ? 1 : 0;
  {
    PROF_BEGIN(KC_INIT);
    k_tree_init<<<32, 256, 0, st>>>(d);
    PROF_END();
  }
  const dim3 bgrid(build_blocks, d.num_groups);
  const int part_blocks = sms * 4;
  // Producer k of the tree (the root build, then split k-1's partition / build) adds into
  // its accumulator; its consumer (the next control step, or the final k_prepare) reads
  // the sum. Over peer memory (xranks > 1) the two alternate by k % 2 (GrowDev::xlocal).
  const bool px = d.xranks > 1;
  const size_t xs = (size_t)d.raw_len + 2;
  auto producer = [&](int k) {
    GrowDev x = d;
    if (px) x.raw = d.xlocal + (size_t)(k & 1) * xs;
    return x;
  };
  auto consumer = [&](int k) {
    GrowDev x = d;
    if (px) {
      x.xpar = k & 1;
      x.raw = d.xlocal + (size_t)((k + 1) & 1) * xs;  // cleared for producer k + 1
    }
    return x;
  };
  auto build = [&](const GrowDev& x, int phase) {
    PROF_BEGIN(KC_BUILD);
    if (x.gh_mode == GH_QPACK)
      q4_kernel(x.q4_shift, x.q4_nch, x.packed4 != 0, x.warp_agg != 0)<<<bgrid, kQ4Threads,
                                                                      build_smem, st>>>(x, phase);
    else if (x.gh_mode == GH_QLUT)
      k_build<GH_QLUT><<<bgrid, kBuildThreads, build_smem, st>>>(x, phase);
    else
      k_build<GH_FLOAT><<<bgrid, kBuildThreads, build_smem, st>>>(x, phase);
    PROF_END();
  };
  // Over peer memory each producer launch publishes its own exchange at its end
  // (producer_signal); without it a one-warp k_xsignal follows. With NCCL the sum
  // follows the producer.
  const bool self_sig = px && d.arrive != nullptr;
  auto exchange = [&](const GrowDev& x) {
    if (px) {
      if (!self_sig) k_xsignal<<<1, 32, 0, st>>>(x);
    } else if (comm) {
      comm->sum_i64(comm->ctx, x.raw, (int64_t)x.raw_len + 1, st);
    }
  };
  {
    GrowDev x = producer(0);
    x.span_slot = kSpanRootBuild;
    x.self_signal = self_sig ? 1 : 0;
    build(x, 0);
    exchange(x);
  }
  // One launch per split on one device: the control step of split s >= 1 runs the main
  // partition of split s - 1 itself when the look-ahead did not (k_fixscan_part). Wide
  // (256-thread) and categorical control steps, peers and the event profiler keep the
  // separate main partition.
  const int ctl_slice = d.slice_end - d.slice_begin;
  const int ctl_grid = std::min(ctl_slice, (d.narrow_scan && !d.has_cat ? 4 : 1) * sms);
  const FixscanPartKernel fpk =
      fixscan_part_kernel(d.q4_shift, d.q4_nch, d.gh_mode == GH_FLOAT, d.packed4 != 0);
  const bool fuse_main = d.fused && la_on && d.fuse_main && !prof && !px && !comm &&
                         !d.has_cat && !d.narrow_scan && fpk != nullptr &&
                         ctl_grid >= d.private_tiles;
  for (int s = 0; s < d.L - 1; ++s) {
    if (la_on && !prof && s >= 2) cudaStreamWaitEvent(st, las->done[(s - 2) & (kLaSlots - 1)], 0);
    if (fuse_main && s >= 1) {
      GrowDev x = consumer(s);
      x.span_slot = span_slot_of(s, SPAN_FIXSCAN);
      GrowDev xp = producer(s);
      xp.span_slot = span_slot_of(s - 1, SPAN_PARTITION);
      x.mainrec = xp.mainrec = d.mainrec;
      const int mg = (s - 1) < las->main_early_steps ? las->main_blocks : las->main_late_blocks;
      fpk<<<std::max(ctl_grid, mg), 1024, fused_partition_smem(), st>>>(x, s, xp, ctl_grid);
    } else {
      GrowDev x = consumer(s);
      x.span_slot = span_slot_of(s, SPAN_FIXSCAN);
      x.mainrec = fuse_main ? d.mainrec : nullptr;  // the first step writes step 1's record
      PROF_BEGIN(KC_FIXSCAN);
      // variants: categorical features, and the peer exchange (off on one device). One
      // CTA per feature of this rank's slice, at most one resident wave of CTAs (each
      // takes features blockIdx.x, blockIdx.x + grid, ...): a CTA applies the pending
      // split once, however many features it scans.
      const int slice = x.slice_end - x.slice_begin;
      const int grid = std::min(slice, (x.narrow_scan && !x.has_cat ? 4 : 1) * sms);
      if (x.has_cat)
        (px ? k_fixscan<true, true, 1024> : k_fixscan<true, false, 1024>)<<<grid, 1024, 0, st>>>(
            x, s);
      else if (x.narrow_scan)  // every feature has at most 64 bins: 256-thread CTAs
        (px ? k_fixscan<false, true, 256> : k_fixscan<false, false, 256>)<<<grid, 256, 0, st>>>(
            x, s);
      else
        (px ? k_fixscan<false, true, 1024> : k_fixscan<false, false, 1024>)<<<grid, 1024, 0, st>>>(
            x, s);
      PROF_END();
    }
    const int phase = s < d.L - 2 ? 1 : 2;
    GrowDev x = producer(s + 1);
    x.span_slot = span_slot_of(s, SPAN_PARTITION);
    x.self_signal = (self_sig && x.fused) ? 1 : 0;  // the fused partition is the producer
    const bool la_step = la_on && s <= d.L - 3;
    // A profiled sequence runs the look-ahead on the main stream, right after the control
    // step: each launch's event span is then its own run, not its wait for free SMs.
    if (la_step && !prof) cudaEventRecord(las->fork, st);
    // the main partition is launched before the look-ahead, so that its CTAs (which
    // mostly find the split already partitioned) are placed first
    if (x.fused && fuse_main && s < d.L - 2) {
      // the next control step partitions this split's leaf when it must
    } else if (x.fused) {
      PROF_BEGIN(KC_PARTITION);
      const int main_grid =
          la_on ? (s < las->main_early_steps ? las->main_blocks : las->main_late_blocks) : sms;
      part_q4_kernel(x.q4_shift, x.q4_nch, x.gh_mode == GH_FLOAT, x.packed4 != 0)<<<main_grid,
                                                                kFpThreads,
                                                                fused_partition_smem(), st>>>(
          x, phase == 1 ? 1 : 0, -1);
      PROF_END();
    } else {
      {
        PROF_BEGIN(KC_PARTITION);
        k_partition<<<part_blocks, kPartThreads, 0, st>>>(x);
        PROF_END();
      }
      GrowDev xb = x;
      xb.span_slot = span_slot_of(s, SPAN_BUILD);
      xb.self_signal = self_sig ? 1 : 0;  // the build after the partition is the producer
      build(xb, phase);
    }
    if (la_step) {
      const cudaStream_t lst = prof ? st : las->st;
      if (!prof) cudaStreamWaitEvent(lst, las->fork, 0);
      const int pslot = prof ? prof->begin(lst, KC_PARTITION) : -1;
      GrowDev xl = x;
      xl.span_slot = span_slot_of(s, SPAN_LOOKAHEAD);
      xl.self_signal = self_sig ? 2 : 0;
      part_q4_kernel(x.q4_shift, x.q4_nch, x.gh_mode == GH_FLOAT, x.packed4 != 0)<<<
          fuse_main ? las->blocks_fused : las->blocks, kFpThreads,
                                                                fused_partition_smem(),
                                                                lst>>>(xl, 1, s & (kLaSlots - 1));
      if (prof) prof->end(lst, pslot);
      if (px && !self_sig) k_lasignal<<<1, 32, 0, lst>>>(x);  // every rank may read the slot
      if (!prof) cudaEventRecord(las->done[s & (kLaSlots - 1)], lst);
    }
    exchange(x);
  }
  // the last split may come from the last look-ahead, which also joins the second stream
  if (la_on && !prof && d.L >= 3)
    cudaStreamWaitEvent(st, las->done[(d.L - 3) & (kLaSlots - 1)], 0);
  {
    PROF_BEGIN(KC_PREPARE);
    k_prepare<<<1, 32, 0, st>>>(consumer(d.L - 1), d.L - 1);
    PROF_END();
  }
}

int q4_max_cells() { return kQ4MaxCells; }

bool q4_supported(int shift, int nch, bool pack4) { return q4_kernel(shift, nch, pack4) != nullptr; }

void set_build_smem_limit(size_t bytes) {
  for (int sh = 4; sh <= 8; ++sh)
    for (int n = 1; n <= 8; ++n)
      for (bool p4 : {false, true})
        for (bool agg : {false, true}) {
          const Q4Kernel k = q4_kernel(sh, n, p4, agg);
          if (!k) continue;
          cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)(4 * sizeof(uint32_t) * kQ4MaxCells));
          cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        }
  for (int sh = 4; sh <= 8; ++sh)
    for (int n = 1; n <= kFpMaxChunks; ++n)
      for (bool f32 : {false, true})
        for (bool p4 : {false, true})
          if (part_q4_kernel(sh, n, f32, p4))
            cudaFuncSetAttribute(part_q4_kernel(sh, n, f32, p4),
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)fused_partition_smem());
  for (int n = 1; n <= 2; ++n)
    for (bool f32 : {false, true})
      cudaFuncSetAttribute(fixscan_part_kernel(8, n, f32, false),
                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)fused_partition_smem());
  cudaFuncSetAttribute(k_build<GH_QLUT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       (int)bytes);
  cudaFuncSetAttribute(k_build<GH_FLOAT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       (int)bytes);
}

void launch_construct_histogram_f32(const uint8_t* bins_rm, int32_t stride, int64_t n,
                                    const float2* gh, int32_t num_bin, double scale_g,
                                    double scale_h, long long* raw, cudaStream_t st) {
  int blocks = (int)std::min<int64_t>((n + 255) / 256, (int64_t)num_sms() * 4);
  if (blocks < 1) blocks = 1;
  k_hist_standalone<<<blocks, 256, 0, st>>>(bins_rm, stride, n, gh, num_bin, scale_g, scale_h,
                                            raw);
}

void launch_scan_features(const double* hist, const DevFeature* feats, int32_t n_feats,
                          DevGainConfig cfg, DevLeafSplits ls, DevSplitInfo* out,
                          cudaStream_t st) {
  if (n_feats <= 0) return;
  k_scan_standalone<<<n_feats, 512, 0, st>>>(hist, feats, cfg, ls, out);
}

void launch_partition_rows(const uint8_t* bins_rm, int32_t stride, int32_t feature,
                           const DevFeature* feat, uint32_t threshold, int32_t default_left,
                           int64_t count, uint32_t* dst, unsigned long long* status,
                           int32_t* left_total, uint32_t* ticket, uint32_t* error,
                           cudaStream_t st) {
  const int32_t ntiles = (int32_t)((count + kPartTile - 1) / kPartTile);
  int blocks = std::min(ntiles, num_sms() * 4);
  if (blocks < 1) blocks = 1;
  k_partition_standalone<<<blocks, kPartThreads, 0, st>>>(
      bins_rm, stride, feature, feat, threshold, default_left, (int32_t)count, dst, status,
      left_total, ticket, error);
}

void launch_gather_partition(const GrowDev& d, uint32_t* out, cudaStream_t st) {
  k_gather_partition<<<dim3(64, d.L), 256, 0, st>>>(d, out);
}

void launch_subtract(const double* parent, const double* child, double* out, int64_t len,
                     cudaStream_t st) {
  int blocks = (int)std::min<int64_t>((len + 255) / 256, 1024);
  if (blocks < 1) blocks = 1;
  k_subtract<<<blocks, 256, 0, st>>>(parent, child, out, len);
}

}  // namespace lgbm_b200
