// Large host <-> device copies through two pinned staging buffers: several host threads
// move pageable memory into one buffer while the DMA engine drains the other.
#include "host_copy.h"

#include <algorithm>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

namespace lgbm_b200 {
namespace {

constexpr size_t kStageBytes = 32ull << 20;  // per pinned buffer
constexpr size_t kPiece = 1ull << 20;        // unit of work of one host thread
constexpr unsigned kMaxCopyThreads = 8;

struct StagePool {
  std::mutex mu;
  void* buf[2] = {nullptr, nullptr};
  bool tried = false;
  bool ok = false;
};

StagePool& pool() {
  static StagePool p;
  return p;
}

// The pinned buffers, allocated on first use and kept for the life of the process
// (portable: any device may DMA from them). False when pinned memory cannot be had.
bool ensure_pool(StagePool& p) {
  if (p.tried) return p.ok;
  p.tried = true;
  for (int k = 0; k < 2; ++k) {
    if (cudaHostAlloc(&p.buf[k], kStageBytes, cudaHostAllocPortable) != cudaSuccess) {
      cudaGetLastError();
      for (int j = 0; j < k; ++j) cudaFreeHost(p.buf[j]);
      p.buf[0] = p.buf[1] = nullptr;
      return false;
    }
  }
  p.ok = true;
  return true;
}

struct Seg {
  char* dst;
  const char* src;
  size_t len;
};

// memcpy of every segment, split into 1 MB pieces dealt round robin to the threads
void parallel_copy(const std::vector<Seg>& segs) {
  std::vector<Seg> pieces;
  for (const Seg& s : segs)
    for (size_t o = 0; o < s.len; o += kPiece)
      pieces.push_back({s.dst + o, s.src + o, std::min(kPiece, s.len - o)});
  const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
  const size_t T = std::min<size_t>(std::min(kMaxCopyThreads, hw), pieces.size());
  auto work = [&](size_t t) {
    for (size_t i = t; i < pieces.size(); i += T)
      std::memcpy(pieces[i].dst, pieces[i].src, pieces[i].len);
  };
  if (T <= 1) {
    work(0);
    return;
  }
  std::vector<std::thread> th;
  th.reserve(T - 1);
  for (size_t t = 1; t < T; ++t) th.emplace_back(work, t);
  work(0);
  for (auto& x : th) x.join();
}

struct Events {
  cudaEvent_t ev[2] = {nullptr, nullptr};
  ~Events() {
    for (cudaEvent_t e : ev)
      if (e) cudaEventDestroy(e);
  }
  cudaError_t create() {
    for (cudaEvent_t& e : ev) {
      const cudaError_t r = cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
      if (r != cudaSuccess) return r;
    }
    return cudaSuccess;
  }
};

#define HC_TRY(x)                              \
  do {                                         \
    const cudaError_t e_ = (x);                \
    if (e_ != cudaSuccess) return e_;          \
  } while (0)

}  // namespace

cudaError_t staged_h2d(void* dst, const void* const* srcs, int nsrc, size_t bytes_each,
                       size_t dst_stride, cudaStream_t st) {
  StagePool& p = pool();
  std::lock_guard<std::mutex> lk(p.mu);
  if (!ensure_pool(p)) {  // the driver stages pageable copies itself
    for (int k = 0; k < nsrc; ++k)
      HC_TRY(cudaMemcpyAsync(static_cast<char*>(dst) + k * dst_stride, srcs[k], bytes_each,
                             cudaMemcpyHostToDevice, st));
    return cudaStreamSynchronize(st);
  }
  Events ev;
  HC_TRY(ev.create());
  bool pending[2] = {false, false};
  int cur = 0;
  size_t fill = 0;
  std::vector<Seg> host, dma;
  auto flush = [&]() -> cudaError_t {
    if (fill == 0) return cudaSuccess;
    parallel_copy(host);
    for (const Seg& s : dma)
      HC_TRY(cudaMemcpyAsync(s.dst, s.src, s.len, cudaMemcpyHostToDevice, st));
    HC_TRY(cudaEventRecord(ev.ev[cur], st));
    pending[cur] = true;
    cur ^= 1;
    fill = 0;
    host.clear();
    dma.clear();
    // the other buffer is written next: its DMA must have finished
    if (pending[cur]) HC_TRY(cudaEventSynchronize(ev.ev[cur]));
    pending[cur] = false;
    return cudaSuccess;
  };
  for (int k = 0; k < nsrc; ++k) {
    size_t off = 0;
    while (off < bytes_each) {
      const size_t n = std::min(bytes_each - off, kStageBytes - fill);
      char* stage = static_cast<char*>(p.buf[cur]) + fill;
      host.push_back({stage, static_cast<const char*>(srcs[k]) + off, n});
      dma.push_back({static_cast<char*>(dst) + k * dst_stride + off, stage, n});
      fill += n;
      off += n;
      if (fill == kStageBytes) HC_TRY(flush());
    }
  }
  HC_TRY(flush());
  // the next call reuses both buffers
  for (int k = 0; k < 2; ++k)
    if (pending[k]) HC_TRY(cudaEventSynchronize(ev.ev[k]));
  return cudaSuccess;
}

cudaError_t staged_d2h(void* dst, const void* src, size_t bytes, cudaStream_t st) {
  StagePool& p = pool();
  std::lock_guard<std::mutex> lk(p.mu);
  if (!ensure_pool(p)) {
    HC_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, st));
    return cudaStreamSynchronize(st);
  }
  Events ev;
  HC_TRY(ev.create());
  size_t issued = 0, copied = 0;
  size_t off[2] = {0, 0}, len[2] = {0, 0};
  auto issue = [&](int b) -> cudaError_t {
    const size_t n = std::min(kStageBytes, bytes - issued);
    HC_TRY(cudaMemcpyAsync(p.buf[b], static_cast<const char*>(src) + issued, n,
                           cudaMemcpyDeviceToHost, st));
    HC_TRY(cudaEventRecord(ev.ev[b], st));
    off[b] = issued;
    len[b] = n;
    issued += n;
    return cudaSuccess;
  };
  if (bytes > 0) HC_TRY(issue(0));
  if (issued < bytes) HC_TRY(issue(1));
  int b = 0;
  while (copied < bytes) {
    HC_TRY(cudaEventSynchronize(ev.ev[b]));
    parallel_copy({{static_cast<char*>(dst) + off[b], static_cast<const char*>(p.buf[b]), len[b]}});
    copied += len[b];
    if (issued < bytes) HC_TRY(issue(b));
    b ^= 1;
  }
  return cudaSuccess;
}

}  // namespace lgbm_b200
