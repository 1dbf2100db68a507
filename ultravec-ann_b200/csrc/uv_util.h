// uv_util.h -- launchers for the record-level utility kernels (util.cu).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "uv_common.cuh"

namespace uvb {

cudaError_t launch_digest(const uint8_t *codes, int stride, int code_bytes, const uint32_t *start,
                          int64_t n, unsigned long long *out, cudaStream_t st);
cudaError_t launch_windows(const uint8_t *codes, int stride, int code_bytes,
                           const uint32_t *start, int64_t n, int dim, int mem, int bits,
                           uint32_t *out, cudaStream_t st);
cudaError_t launch_decode(const uint32_t *windows, const float *code, int64_t n,
                          const RotParams &rot, float *out, cudaStream_t st);
cudaError_t launch_rotate(const float *rows, int64_t n, const RotParams &rot, float *out,
                          cudaStream_t st);

}  // namespace uvb
