// Large copies between pageable host memory and the device through pinned staging.
#pragma once

#include <cstddef>
#include <cuda_runtime.h>

namespace lgbm_b200 {

// Copies nsrc host ranges of `bytes_each` bytes (srcs[k]) to dst + k * dst_stride on the
// device, in stream order on `st`. Several host threads copy each chunk of the sources
// into a pinned buffer while the DMA of the previous chunk runs; two pinned buffers are
// kept for the life of the process. The sources may be reused when the call returns.
cudaError_t staged_h2d(void* dst, const void* const* srcs, int nsrc, size_t bytes_each,
                       size_t dst_stride, cudaStream_t st);

// Copies `bytes` from the device (after the work already queued on `st`) into pageable
// host memory; returns when the data is in `dst`.
cudaError_t staged_d2h(void* dst, const void* src, size_t bytes, cudaStream_t st);

}  // namespace lgbm_b200
