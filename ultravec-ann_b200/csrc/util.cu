// util.cu -- record-level device kernels of the codec API: encode_digest,
// window_at over whole records, decode_codes, and the bare rotation.
#include "uv_kernels.h"
#include "uv_team.cuh"
#include "uv_util.h"

namespace uvb {

// encode_digest (src/trellis.rs:970-990): per record FNV-1a over the four
// little-endian bytes of start, then the code bytes; XOR-folded.
__global__ void digest_kernel(const uint8_t *codes, int stride, int code_bytes,
                              const uint32_t *start, int64_t n, unsigned long long *out) {
  unsigned long long acc = 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    uint64_t h = 0xcbf29ce484222325ULL;
    const uint32_t st = start[i];
    for (int b = 0; b < 4; b++) {
      h ^= (uint64_t)((st >> (8 * b)) & 0xffu);
      h *= 0x00000100000001b3ULL;
    }
    const uint8_t *c = codes + i * (int64_t)stride;
    for (int b = 0; b < code_bytes; b++) {
      h ^= (uint64_t)c[b];
      h *= 0x00000100000001b3ULL;
    }
    acc ^= h;
  }
  for (int o = 16; o > 0; o >>= 1) acc ^= __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) atomicXor(out, acc);
}

// windows_into (src/trellis.rs:1576-1600) for each record: the (M+B)-bit
// field at offset i*B of [start (M bits) || codes], MSB first.
__global__ void windows_kernel(const uint8_t *codes, int stride, int code_bytes,
                               const uint32_t *start, int64_t n, int dim, int mem, int bits,
                               uint32_t *out) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n) return;
  const uint32_t width = (uint32_t)(mem + bits);
  const uint64_t wmask = (1ull << width) - 1;
  uint64_t acc = start[r];
  uint32_t nbits = (uint32_t)mem;
  int byte = 0;
  const uint8_t *c = codes + r * (int64_t)stride;
  for (int i = 0; i < dim; i++) {
    while (nbits < width && byte < code_bytes) {
      acc = (acc << 8) | c[byte];
      nbits += 8;
      byte++;
    }
    if (nbits < width) {
      acc <<= (width - nbits);
      nbits = width;
    }
    out[r * dim + i] = (uint32_t)((acc >> (nbits - width)) & wmask);
    nbits -= (uint32_t)bits;
    acc &= (1ull << nbits) - 1;
  }
}

// decode_codes (src/trellis.rs:705-720): table values by window, then the
// inverse rotation; one warp per record.
__global__ void decode_kernel(const uint32_t *windows, const float *code, int64_t n,
                              RotParams rot, int dim_pad, float *out) {
  extern __shared__ __align__(16) float smem[];
  const int team = threadIdx.x >> 5;
  Team tm;
  tm.T = 32;
  tm.cta = false;
  tm.t = threadIdx.x & 31;
  float *x = smem + (size_t)team * dim_pad;
  const int d = rot.dim;
  const int64_t iters = (n + (int64_t)gridDim.x * 8 - 1) / ((int64_t)gridDim.x * 8);
  for (int64_t it = 0; it < iters; it++) {
    const int64_t r = ((int64_t)it * gridDim.x + blockIdx.x) * 8 + team;
    const bool valid = r < n;
    const int64_t rr = valid ? r : n - 1;
    for (int i = tm.t; i < d; i += 32) x[i] = code[windows[rr * d + i]];
    tm.sync();
    team_rotate(x, rot, tm, true);
    if (valid)
      for (int i = tm.t; i < d; i += 32) out[rr * d + i] = x[i];
    tm.sync();
  }
}

// Rotation::apply of raw rows (src/lib.rs:472-484); one warp per row.
__global__ void rotate_kernel(const float *rows, int64_t n, RotParams rot, int dim_pad,
                              float *out) {
  extern __shared__ __align__(16) float smem[];
  const int team = threadIdx.x >> 5;
  Team tm;
  tm.T = 32;
  tm.cta = false;
  tm.t = threadIdx.x & 31;
  float *x = smem + (size_t)team * dim_pad;
  const int d = rot.dim;
  const int64_t iters = (n + (int64_t)gridDim.x * 8 - 1) / ((int64_t)gridDim.x * 8);
  for (int64_t it = 0; it < iters; it++) {
    const int64_t r = ((int64_t)it * gridDim.x + blockIdx.x) * 8 + team;
    const bool valid = r < n;
    const int64_t rr = valid ? r : n - 1;
    for (int i = tm.t; i < d; i += 32) x[i] = rows[rr * d + i];
    tm.sync();
    team_rotate(x, rot, tm, false);
    if (valid)
      for (int i = tm.t; i < d; i += 32) out[rr * d + i] = x[i];
    tm.sync();
  }
}

cudaError_t launch_digest(const uint8_t *codes, int stride, int code_bytes, const uint32_t *start,
                          int64_t n, unsigned long long *out, cudaStream_t st) {
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 4096));
  digest_kernel<<<grid, 256, 0, st>>>(codes, stride, code_bytes, start, n, out);
  return cudaGetLastError();
}

cudaError_t launch_windows(const uint8_t *codes, int stride, int code_bytes,
                           const uint32_t *start, int64_t n, int dim, int mem, int bits,
                           uint32_t *out, cudaStream_t st) {
  const int grid = (int)((n + 127) / 128);
  windows_kernel<<<grid, 128, 0, st>>>(codes, stride, code_bytes, start, n, dim, mem, bits, out);
  return cudaGetLastError();
}

static int row_grid(int64_t n) {
  return (int)std::max<int64_t>(1, std::min<int64_t>((n + 7) / 8, 148 * 16));
}

cudaError_t launch_decode(const uint32_t *windows, const float *code, int64_t n,
                          const RotParams &rot, float *out, cudaStream_t st) {
  const int dim_pad = (rot.dim + 3) & ~3;
  const size_t smem = (size_t)dim_pad * 4 * 8;
  cudaError_t e = cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  decode_kernel<<<row_grid(n), 256, smem, st>>>(windows, code, n, rot, dim_pad, out);
  return cudaGetLastError();
}

cudaError_t launch_rotate(const float *rows, int64_t n, const RotParams &rot, float *out,
                          cudaStream_t st) {
  const int dim_pad = (rot.dim + 3) & ~3;
  const size_t smem = (size_t)dim_pad * 4 * 8;
  cudaError_t e = cudaFuncSetAttribute(rotate_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  rotate_kernel<<<row_grid(n), 256, smem, st>>>(rows, n, rot, dim_pad, out);
  return cudaGetLastError();
}

}  // namespace uvb
