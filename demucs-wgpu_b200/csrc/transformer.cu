// Cross-transformer kernels that are not GEMMs:
//  * layer_norm: nn.LayerNorm(512) per token (ops.rs:596-621), optionally
//    adding a positional table (host.rs:878-890);
//  * group_norm_apply: MyGroupNorm(1, 512) over the whole (tokens, 512) plane
//    per segment from f64 moments accumulated by the producing GEMM
//    (host.rs:1137-1196);
//  * flash_attention: softmax(q k^T / 8) v for 8 heads of 64 with an online
//    softmax, never materialising the score matrix (host.rs:1199-1312,
//    ops.rs:1350-1458).
#include <cuda_bf16.h>

#include "common.cuh"
#include "kernels.h"

#include <algorithm>

namespace dmx {

namespace {

// One warp per token of 512 channels.
__global__ void layer_norm_kernel(const float* __restrict__ x, int64_t rows, int ntok,
                                  const float* __restrict__ w, const float* __restrict__ b,
                                  const float* __restrict__ pos, float* __restrict__ out,
                                  int round_out, uint16_t* __restrict__ out16) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  const float* in = x + row * 512;
  float v[16];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 q = *reinterpret_cast<const float4*>(in + lane * 4 + i * 128);
    v[4 * i] = q.x;
    v[4 * i + 1] = q.y;
    v[4 * i + 2] = q.z;
    v[4 * i + 3] = q.w;
  }
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) s += v[i];
  const float mean = warp_sum(s) / 512.0f;
  float var = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) var += (v[i] - mean) * (v[i] - mean);
  var = warp_sum(var) / 512.0f;
  const float inv = 1.0f / sqrtf(var + 1e-5f);
  float* o = out + row * 512;
  const float* pr = pos ? pos + (row % ntok) * 512 : nullptr;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = lane * 4 + i * 128;
    const float4 w4 = __ldg(reinterpret_cast<const float4*>(w + c));
    const float4 b4 = __ldg(reinterpret_cast<const float4*>(b + c));
    float4 r;
    r.x = (v[4 * i] - mean) * inv * w4.x + b4.x;
    r.y = (v[4 * i + 1] - mean) * inv * w4.y + b4.y;
    r.z = (v[4 * i + 2] - mean) * inv * w4.z + b4.z;
    r.w = (v[4 * i + 3] - mean) * inv * w4.w + b4.w;
    if (pr) {
      const float4 p4 = __ldg(reinterpret_cast<const float4*>(pr + c));
      r.x += p4.x;
      r.y += p4.y;
      r.z += p4.z;
      r.w += p4.w;
    }
    if (out16) {  // the output feeds only bf16 GEMMs: stored as bf16
      const __nv_bfloat162 lo = __float22bfloat162_rn(make_float2(r.x, r.y));
      const __nv_bfloat162 hi = __float22bfloat162_rn(make_float2(r.z, r.w));
      uint2 u;
      u.x = *reinterpret_cast<const uint32_t*>(&lo);
      u.y = *reinterpret_cast<const uint32_t*>(&hi);
      *reinterpret_cast<uint2*>(out16 + row * 512 + c) = u;
      continue;
    }
    if (round_out) {  // the output feeds only tf32 GEMMs: round to nearest here, once
      r.x = round_tf32(r.x);
      r.y = round_tf32(r.y);
      r.z = round_tf32(r.z);
      r.w = round_tf32(r.w);
    }
    *reinterpret_cast<float4*>(o + c) = r;
  }
}

__global__ void group_norm_apply_kernel(float* __restrict__ x, int64_t ntok,
                                        const double* __restrict__ stats,
                                        const float* __restrict__ w, const float* __restrict__ b) {
  const int bi = blockIdx.y;
  const RowNorm rn = row_norm(stats, bi, (double)ntok * 512.0);
  float* base = x + (int64_t)bi * ntok * 512;
  for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4; i < ntok * 512;
       i += (int64_t)gridDim.x * blockDim.x * 4) {
    const int c = (int)(i & 511);
    float4 v = *reinterpret_cast<float4*>(base + i);
    const float4 w4 = __ldg(reinterpret_cast<const float4*>(w + c));
    const float4 b4 = __ldg(reinterpret_cast<const float4*>(b + c));
    float sc, sh;
    sc = rn.inv * w4.x; sh = b4.x - rn.mean * sc; v.x = v.x * sc + sh;
    sc = rn.inv * w4.y; sh = b4.y - rn.mean * sc; v.y = v.y * sc + sh;
    sc = rn.inv * w4.z; sh = b4.z - rn.mean * sc; v.z = v.z * sc + sh;
    sc = rn.inv * w4.w; sh = b4.w - rn.mean * sc; v.w = v.w * sc + sh;
    *reinterpret_cast<float4*>(base + i) = v;
  }
}

// Flash attention, fp32 SIMT. One CTA = 64 queries of one (segment, head);
// 256 threads each own 4 query rows x 4 key columns of the score tile and
// 4 rows x 4 dims of the output.
constexpr int AQ = 64, AK = 64, AD = 64;
__global__ void __launch_bounds__(256) flash_attention_kernel(
    const float* __restrict__ q, int ldq, const float* __restrict__ k, const float* __restrict__ v,
    int ldkv, float* __restrict__ o, int ldo, int nq, int nk, float scale) {
  extern __shared__ float sm[];
  float* Qs = sm;                   // [AD][AQ + 4]   (transposed)
  float* Ks = Qs + AD * (AQ + 4);   // [AD][AK + 4]   (transposed)
  float* Vs = Ks + AD * (AK + 4);   // [AK][AD]
  float* Ps = Vs + AK * AD;         // [AK][AQ + 4]   (transposed)
  const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
  const int q0 = blockIdx.x * AQ, h = blockIdx.y, b = blockIdx.z;
  const float* qb = q + ((int64_t)b * nq) * ldq + h * AD;
  const float* kb = k + ((int64_t)b * nk) * ldkv + h * AD;
  const float* vb = v + ((int64_t)b * nk) * ldkv + h * AD;
  for (int e = tid; e < AQ * AD / 4; e += 256) {
    const int r = e / (AD / 4), c = (e % (AD / 4)) * 4;
    float4 val = make_float4(0.f, 0.f, 0.f, 0.f);
    if (q0 + r < nq) val = *reinterpret_cast<const float4*>(qb + (int64_t)(q0 + r) * ldq + c);
    Qs[(c + 0) * (AQ + 4) + r] = val.x * scale;
    Qs[(c + 1) * (AQ + 4) + r] = val.y * scale;
    Qs[(c + 2) * (AQ + 4) + r] = val.z * scale;
    Qs[(c + 3) * (AQ + 4) + r] = val.w * scale;
  }
  float m[4], l[4], acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  }
  for (int k0 = 0; k0 < nk; k0 += AK) {
    __syncthreads();
    for (int e = tid; e < AK * AD / 4; e += 256) {
      const int r = e / (AD / 4), c = (e % (AD / 4)) * 4;
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
      if (k0 + r < nk) {
        kv = *reinterpret_cast<const float4*>(kb + (int64_t)(k0 + r) * ldkv + c);
        vv = *reinterpret_cast<const float4*>(vb + (int64_t)(k0 + r) * ldkv + c);
      }
      Ks[(c + 0) * (AK + 4) + r] = kv.x;
      Ks[(c + 1) * (AK + 4) + r] = kv.y;
      Ks[(c + 2) * (AK + 4) + r] = kv.z;
      Ks[(c + 3) * (AK + 4) + r] = kv.w;
      *reinterpret_cast<float4*>(Vs + r * AD + c) = vv;
    }
    __syncthreads();
    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
#pragma unroll 8
    for (int d = 0; d < AD; ++d) {
      const float4 a = *reinterpret_cast<const float4*>(Qs + d * (AQ + 4) + ty * 4);
      const float4 c = *reinterpret_cast<const float4*>(Ks + d * (AK + 4) + tx * 4);
      const float av[4] = {a.x, a.y, a.z, a.w}, cv[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) s[i][j] = fmaf(av[i], cv[j], s[i][j]);
    }
    // online softmax over the 16 threads sharing these rows (one half-warp)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (k0 + tx * 4 + j < nk) mx = fmaxf(mx, s[i][j]);
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float mnew = fmaxf(m[i], mx);
      const float corr = expf(m[i] - mnew);
      float rs = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float pv = (k0 + tx * 4 + j < nk) ? expf(s[i][j] - mnew) : 0.f;
        s[i][j] = pv;
        rs += pv;
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, off);
      l[i] = l[i] * corr + rs;
      m[i] = mnew;
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] *= corr;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) Ps[(tx * 4 + j) * (AQ + 4) + ty * 4 + i] = s[i][j];
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < AK; ++kk) {
      const float4 pa = *reinterpret_cast<const float4*>(Ps + kk * (AQ + 4) + ty * 4);
      const float4 vv = *reinterpret_cast<const float4*>(Vs + kk * AD + tx * 4);
      const float pv[4] = {pa.x, pa.y, pa.z, pa.w}, vw[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(pv[i], vw[j], acc[i][j]);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = q0 + ty * 4 + i;
    if (r >= nq) continue;
    const float inv = l[i] > 0.f ? 1.0f / l[i] : 0.f;
    float4 out;
    out.x = acc[i][0] * inv;
    out.y = acc[i][1] * inv;
    out.z = acc[i][2] * inv;
    out.w = acc[i][3] * inv;
    *reinterpret_cast<float4*>(o + ((int64_t)b * nq + r) * ldo + h * AD + tx * 4) = out;
  }
}

}  // namespace

void launch_layer_norm(const float* x, int64_t rows, int ntok, const float* w, const float* b,
                       const float* pos, float* out, cudaStream_t s, bool round_out,
                       uint16_t* out16) {
  layer_norm_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, s>>>(x, rows, ntok, w, b, pos, out,
                                                               round_out ? 1 : 0, out16);
}

void launch_group_norm_apply(float* x, int B, int64_t ntok, const double* stats, const float* w,
                             const float* b, cudaStream_t s) {
  group_norm_apply_kernel<<<dim3(148, B), 256, 0, s>>>(x, ntok, stats, w, b);
}

void launch_flash_attention(const float* q, int ldq, const float* k, const float* v, int ldkv,
                            float* o, int ldo, int B, int heads, int nq, int nk, float scale,
                            cudaStream_t s) {
  const size_t smem = sizeof(float) * (AD * (AQ + 4) + AD * (AK + 4) + AK * AD + AK * (AQ + 4));
  static PerDevice configured;
  if (configured.first())
    cudaFuncSetAttribute(flash_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
  flash_attention_kernel<<<dim3((nq + AQ - 1) / AQ, heads, B), 256, smem, s>>>(
      q, ldq, k, v, ldkv, o, ldo, nq, nk, scale);
}

}  // namespace dmx
