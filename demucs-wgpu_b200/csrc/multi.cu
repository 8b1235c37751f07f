// Boundary merge of the multi-GPU track driver (dmx_separate_track_multi):
// a rank's overlap-add accumulator receives its left neighbour's tail (the
// last chunk's samples past the neighbour's own span) and adds it in. Every
// sample gets at most two weighted contributions, so (a + b) here equals the
// single-GPU driver's (b + a) bit for bit.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace dmx {

namespace {

// acc[r * ld + c] += tail[r * width + c] for r < rows, c < width
__global__ void tail_add_kernel(float* __restrict__ acc, int64_t ld, const float* __restrict__ tail,
                                int64_t width, int rows) {
  const int64_t n = width * rows;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / width, c = i - r * width;
    acc[r * ld + c] += tail[i];
  }
}

}  // namespace

void launch_tail_add(float* acc, int64_t ld, const float* tail, int64_t width, int rows,
                     cudaStream_t s) {
  const int64_t n = width * rows;
  if (n <= 0) return;
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 148 * 8);
  tail_add_kernel<<<blocks, 256, 0, s>>>(acc, ld, tail, width, rows);
}

}  // namespace dmx
