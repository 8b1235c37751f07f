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

// dst[r * dld + c] (+)= src[r * sld + c] for the grid's row r, c < width; 16-byte
// loads and stores wherever both rows share their alignment. `src` may be a
// peer GPU's memory mapped into this process (NVLink loads by the SMs).
template <bool ADD>
__global__ void rows_kernel(float* __restrict__ dst, int64_t dld, const float* __restrict__ src,
                            int64_t sld, int64_t width) {
  float* d = dst + (int64_t)blockIdx.y * dld;
  const float* s = src + (int64_t)blockIdx.y * sld;
  const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nth = (int64_t)gridDim.x * blockDim.x;
  int64_t head = (int64_t)(((16 - (reinterpret_cast<uintptr_t>(d) & 15)) & 15) / 4);
  if (head > width) head = width;
  const bool vec = (reinterpret_cast<uintptr_t>(s + head) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(d) & 3) == 0;
  if (!vec) head = width;  // no common alignment: every element one by one
  for (int64_t i = t0; i < head; i += nth) d[i] = ADD ? __fadd_rn(d[i], s[i]) : s[i];
  const int64_t body = (width - head) / 4;
  float4* d4 = reinterpret_cast<float4*>(d + head);
  const float4* s4 = reinterpret_cast<const float4*>(s + head);
  for (int64_t i = t0; i < body; i += nth) {
    float4 v = s4[i];
    if (ADD) {
      const float4 a = d4[i];
      v = make_float4(__fadd_rn(a.x, v.x), __fadd_rn(a.y, v.y), __fadd_rn(a.z, v.z),
                      __fadd_rn(a.w, v.w));
    }
    d4[i] = v;
  }
  for (int64_t i = head + 4 * body + t0; i < width; i += nth) d[i] = ADD ? __fadd_rn(d[i], s[i]) : s[i];
}

}  // namespace

void launch_rows(bool add, float* dst, int64_t dld, const float* src, int64_t sld, int rows,
                 int64_t width, cudaStream_t s) {
  if (rows <= 0 || width <= 0) return;
  const dim3 grid((unsigned)std::min<int64_t>((width / 4 + 255) / 256 + 1, 1184 / rows + 1),
                  (unsigned)rows);
  if (add)
    rows_kernel<true><<<grid, 256, 0, s>>>(dst, dld, src, sld, width);
  else
    rows_kernel<false><<<grid, 256, 0, s>>>(dst, dld, src, sld, width);
}

void launch_tail_add(float* acc, int64_t ld, const float* tail, int64_t width, int rows,
                     cudaStream_t s) {
  const int64_t n = width * rows;
  if (n <= 0) return;
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 148 * 8);
  tail_add_kernel<<<blocks, 256, 0, s>>>(acc, ld, tail, width, rows);
}

}  // namespace dmx
