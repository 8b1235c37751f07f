// Fixed-order reductions of per-segment moments.
//
// The GroupNorm / normalisation statistics of the forward are sums over one
// segment's values (demucs/ops.rs:564-578, host.rs:1137-1196). Producers
// write one partial (sum, sum of squares) per output position and column slot
// instead of adding into a shared total, and these kernels add the partials
// of each statistic row in an order fixed by the position inside that row. A
// segment's moments then depend neither on scheduling nor on which other
// segments share the launch, so batching chunks differently, or spreading
// them over GPUs, leaves every output bit unchanged.
#include "common.cuh"
#include "kernels.h"

namespace dmx {

namespace {

constexpr int kReduceThreads = 256;

// stats[row] = sum over positions p of the row, then slots, of part[p][slot];
// thread t takes positions t, t + 256, ... of its row in increasing order,
// then the block combines the 256 per-thread sums in a fixed tree.
__global__ void __launch_bounds__(kReduceThreads)
    row_stats_reduce_kernel(const double* __restrict__ part, int nslots, int64_t rowlen,
                            double* __restrict__ stats) {
  __shared__ double red[2][kReduceThreads / 32];
  const int64_t row = blockIdx.x;
  const double* base = part + row * rowlen * nslots * 2;
  double s = 0.0, q = 0.0;
  for (int64_t p = threadIdx.x; p < rowlen; p += kReduceThreads) {
    const double* e = base + p * nslots * 2;
    for (int k = 0; k < nslots; ++k) {
      s += e[2 * k];
      q += e[2 * k + 1];
    }
  }
  s = warp_sum(s);
  q = warp_sum(q);
  if ((threadIdx.x & 31) == 0) {
    red[0][threadIdx.x / 32] = s;
    red[1][threadIdx.x / 32] = q;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double ts = 0.0, tq = 0.0;
    for (int w = 0; w < kReduceThreads / 32; ++w) {
      ts += red[0][w];
      tq += red[1][w];
    }
    stats[2 * row] = ts;
    stats[2 * row + 1] = tq;
  }
}

// stats[row] = sum over k < nparts of part[row][k], in increasing k.
__global__ void sum_partials_kernel(const double* __restrict__ part, int nparts, int rows,
                                    double* __restrict__ stats) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  const double* e = part + (int64_t)row * nparts * 2;
  double s = 0.0, q = 0.0;
  for (int k = 0; k < nparts; ++k) {
    s += e[2 * k];
    q += e[2 * k + 1];
  }
  stats[2 * row] = s;
  stats[2 * row + 1] = q;
}

}  // namespace

void launch_row_stats_reduce(const double* part, int nslots, int64_t rowlen, int rows,
                             double* stats, cudaStream_t s) {
  if (rows <= 0) return;
  row_stats_reduce_kernel<<<rows, kReduceThreads, 0, s>>>(part, nslots, rowlen, stats);
}

void launch_sum_partials(const double* part, int nparts, int rows, double* stats, cudaStream_t s) {
  if (rows <= 0) return;
  sum_partials_kernel<<<(rows + 127) / 128, 128, 0, s>>>(part, nparts, rows, stats);
}

}  // namespace dmx
