// Bag of networks (htdemucs_ft): the per-source weighted combination of the
// networks' outputs, BagCombineForward::start (api.rs:319-361) and the bag
// branch of Demucs::collect (api.rs:894-969).
//
// For each source s the reference starts from zeros and, for every network k
// in bag order whose weight w[k][s] is nonzero (and s is requested), adds the
// lane out_k[s] * w[k][s] (the product rounded to f32 first, then the sum),
// then divides by the f32 sum of those weights. The kernel forms exactly the
// same roundings (__fmul_rn / __fadd_rn / __fdiv_rn, no contraction into an
// FMA), so the combination itself is bit-identical to the reference's. Lanes
// of sources that are not requested are written as zeros, as the reference's
// `combined` array leaves them.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace dmx {

namespace {

__global__ void bag_combine_kernel(BagTerms t, int64_t lane, int64_t total_lanes,
                                   float* __restrict__ out) {
  // one thread per 4 consecutive floats of one lane (lane % 4 == 0 here)
  const int64_t quads = total_lanes * (lane / 4);
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < quads;
       q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t li = q / (lane / 4);        // (segment, source, channel) lane index
    const int s = (int)((li / t.channels) % t.sources);
    const int64_t off = li * lane + (q - li * (lane / 4)) * 4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < t.count[s]; ++j) {
      const float w = t.weight[s][j];
      const float4 v = __ldg(reinterpret_cast<const float4*>(t.out[t.net[s][j]] + off));
      acc.x = __fadd_rn(acc.x, __fmul_rn(v.x, w));
      acc.y = __fadd_rn(acc.y, __fmul_rn(v.y, w));
      acc.z = __fadd_rn(acc.z, __fmul_rn(v.z, w));
      acc.w = __fadd_rn(acc.w, __fmul_rn(v.w, w));
    }
    if (t.count[s] > 0) {
      const float tot = t.total[s];
      acc.x = __fdiv_rn(acc.x, tot);
      acc.y = __fdiv_rn(acc.y, tot);
      acc.z = __fdiv_rn(acc.z, tot);
      acc.w = __fdiv_rn(acc.w, tot);
    }
    *reinterpret_cast<float4*>(out + off) = acc;
  }
}

// The same for lanes whose length is not a multiple of 4 floats.
__global__ void bag_combine_scalar_kernel(BagTerms t, int64_t lane, int64_t total_lanes,
                                          float* __restrict__ out) {
  const int64_t n = total_lanes * lane;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t li = i / lane;
    const int s = (int)((li / t.channels) % t.sources);
    float acc = 0.f;
    for (int j = 0; j < t.count[s]; ++j)
      acc = __fadd_rn(acc, __fmul_rn(__ldg(t.out[t.net[s][j]] + i), t.weight[s][j]));
    out[i] = t.count[s] > 0 ? __fdiv_rn(acc, t.total[s]) : acc;
  }
}

}  // namespace

void launch_bag_combine(const BagTerms& t, int64_t segments, int64_t samples, float* out,
                        cudaStream_t s) {
  const int64_t lanes = segments * t.sources * t.channels;
  const int threads = 256;
  const int64_t work = samples % 4 == 0 ? lanes * (samples / 4) : lanes * samples;
  // enough blocks to cover the work, capped at 148 SMs x 8 resident blocks
  const int blocks = (int)std::min<int64_t>((work + threads - 1) / threads, 148 * 8);
  if (blocks <= 0) return;
  if (samples % 4 == 0)
    bag_combine_kernel<<<blocks, threads, 0, s>>>(t, samples, lanes, out);
  else
    bag_combine_scalar_kernel<<<blocks, threads, 0, s>>>(t, samples, lanes, out);
}

}  // namespace dmx
