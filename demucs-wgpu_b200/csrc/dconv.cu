// DConv residual branch, fused (host.rs:985-1059; ops.rs:930-1094 for the
// fused GroupNorm + GLU + LayerScale tail). Per DConv layer d (dilation 2^d):
//
//   y = conv1(x)                  k = 3, C -> hid = C/8, padding = dilation
//   g = GELU(GroupNorm1(y))       one group over (hid, T) per row
//   z = conv2(g)                  1x1, hid -> 2C
//   x += gamma * GLU(GroupNorm1(z))   one group over (2C, T) per row
//
// x is channels-last (rows, T, C) and is updated in place; a row is one
// (batch, frequency) line of the spectral branch or one batch item of the
// waveform branch.
//
// Rows of at most kTile positions (the spectral branch: T = 336 frames) run in
// ONE launch, one CTA per row: conv1 over the row, the row's moments reduced
// in the CTA, g kept in shared memory, the moments of z taken from g alone
// (sum z = v.g~, sum z^2 = g~'Mg~ with host-side v, M: z_moments below), then z
// formed once, for the output — x crosses HBM once each way (its second read,
// for the residual, comes from L2). Longer rows (the waveform branch) are
// tiled in three launches: conv1 + per-tile moments (y to HBM: C/8 channels),
// z moments per tile, then the output; each tile reduces its row's per-tile
// moments in a fixed order, so the result does not depend on scheduling.
//
// Arithmetic is fp32 with f64 moment sums (the reference's GroupNorm
// accumulates in f64, ops.rs:930-1094); every build precision uses it.

#include <cstdint>

#include "common.cuh"
#include "kernels.h"

namespace dmx {
namespace {

constexpr int kThreads = 384;  // a multiple of every C (48, 96, 192, 384) and of 32
constexpr int kWarps = kThreads / 32;
constexpr int kTile = 384;     // positions per tile
constexpr int kCC = 16;        // conv1 input channels staged per step
constexpr int kMaxDil = 2;

template <int C>
struct Dc {
  static constexpr int HID = C / 8;
  static constexpr int HIDP = (HID + 3) / 4 * 4;  // g row stride in shared memory
  // conv1: thread (hg, pg) computes HN hidden channels of PM positions
  static constexpr int HN = HID <= 24 ? 6 : 12;
  static constexpr int HG = HID / HN;
  static constexpr int PG = kThreads / HG;
  static constexpr int PM = kTile / PG;
  // conv2: thread (g0, c) computes channel c of every G-th position
  static constexpr int G = kThreads / C;
  static constexpr int XS = (kTile + 2 * kMaxDil) * (kCC + 1);
  static constexpr int WS = 3 * kCC * HID;
  static constexpr int YS = kTile * HIDP;
  static_assert(HID % HN == 0 && kThreads % HG == 0 && kTile % PG == 0, "conv1 tiling");
  static_assert(kThreads % C == 0 && C % kCC == 0, "conv2 tiling");
};

DMX_DEVICE void warp_sum2(double& s, double& q) {
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, o);
    q += __shfl_xor_sync(0xffffffffu, q, o);
  }
}

// CTA-wide sum of (s, q) in a fixed order; every thread gets the result.
DMX_DEVICE void block_sum2(double& s, double& q, double* red) {
  warp_sum2(s, q);
  __syncthreads();  // red may still be read by a previous reduction
  if ((threadIdx.x & 31) == 0) {
    red[2 * (threadIdx.x >> 5)] = s;
    red[2 * (threadIdx.x >> 5) + 1] = q;
  }
  __syncthreads();
  s = 0.0;
  q = 0.0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    s += red[2 * w];
    q += red[2 * w + 1];
  }
}

// Sum of a row's per-tile moments (fixed order) -> GroupNorm mean, 1/std.
DMX_DEVICE void row_moments(const double* part, int tiles, double count, float& mean, float& inv,
                            double* red) {
  if (threadIdx.x < 32) {
    double s = 0.0, q = 0.0;
    for (int i = threadIdx.x; i < tiles; i += 32) {
      s += part[2 * i];
      q += part[2 * i + 1];
    }
    warp_sum2(s, q);
    if (threadIdx.x == 0) {
      red[0] = s;
      red[1] = q;
    }
  }
  __syncthreads();
  const double m = red[0] / count;
  const double var = fmax(red[1] / count - m * m, 0.0);
  mean = (float)m;
  inv = 1.0f / (float)sqrt(var + 1e-5);
}

DMX_DEVICE void moments_to_norm(double s, double q, double count, float& mean, float& inv) {
  const double m = s / count;
  const double var = fmax(q / count - m * m, 0.0);
  mean = (float)m;
  inv = 1.0f / (float)sqrt(var + 1e-5);
}

// conv1 of positions [t0, t0 + kTile) of one row (positions >= T read zeros
// and are discarded by the caller). acc[i][j]: hidden channel hg*HN + j of
// position pg + i*PG, bias included.
template <int C>
DMX_DEVICE void conv1_tile(const float* __restrict__ xr, int T, int t0, int dil,
                           const DConvArgs& a, float* xs, float* ws,
                           float2 (&acc)[Dc<C>::PM][Dc<C>::HN / 2]) {
  using S = Dc<C>;
  const int tid = threadIdx.x, hg = tid / S::PG, pg = tid % S::PG;
#pragma unroll
  for (int j = 0; j < S::HN / 2; ++j) {
    const float2 b = make_float2(a.b1[hg * S::HN + 2 * j], a.b1[hg * S::HN + 2 * j + 1]);
#pragma unroll
    for (int i = 0; i < S::PM; ++i) acc[i][j] = b;
  }
  const int xrows = kTile + 2 * dil;
  for (int c0 = 0; c0 < C; c0 += kCC) {
    __syncthreads();  // the previous chunk is consumed
    for (int i = tid; i < xrows * kCC; i += kThreads) {
      const int r = i / kCC, cc = i - r * kCC;
      const int t = t0 - dil + r;
      xs[r * (kCC + 1) + cc] = (t >= 0 && t < T) ? xr[(int64_t)t * C + c0 + cc] : 0.f;
    }
    for (int i = tid; i < S::WS; i += kThreads) {
      const int h = i % S::HID, kc = i / S::HID;
      const int k = kc / kCC, cc = kc - k * kCC;
      ws[i] = a.w1[(int64_t)(k * C + c0 + cc) * a.w1_ld + h];
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const float* xk = xs + (pg + k * dil) * (kCC + 1);
#pragma unroll 4
      for (int cc = 0; cc < kCC; ++cc) {
        float xv[S::PM];
#pragma unroll
        for (int i = 0; i < S::PM; ++i) xv[i] = xk[i * S::PG * (kCC + 1) + cc];
        const float2* wr = reinterpret_cast<const float2*>(ws + (k * kCC + cc) * S::HID + hg * S::HN);
        float2 wv[S::HN / 2];
#pragma unroll
        for (int j = 0; j < S::HN / 2; ++j) wv[j] = wr[j];
#pragma unroll
        for (int i = 0; i < S::PM; ++i) {
          const float2 xx = make_float2(xv[i], xv[i]);
#pragma unroll
          for (int j = 0; j < S::HN / 2; ++j) acc[i][j] = __ffma2_rn(xx, wv[j], acc[i][j]);
        }
      }
    }
  }
}

// f64 moments of the valid conv1 outputs of this thread.
template <int C>
DMX_DEVICE void conv1_moments(const float2 (&acc)[Dc<C>::PM][Dc<C>::HN / 2], int np, double& s,
                              double& q) {
  using S = Dc<C>;
  const int pg = threadIdx.x % S::PG;
  s = 0.0;
  q = 0.0;
#pragma unroll
  for (int i = 0; i < S::PM; ++i) {
    if (pg + i * S::PG < np) {
#pragma unroll
      for (int j = 0; j < S::HN / 2; ++j) {
        const double v0 = acc[i][j].x, v1 = acc[i][j].y;
        s += v0 + v1;
        q += v0 * v0 + v1 * v1;
      }
    }
  }
}

// g = GELU(GroupNorm1(y)) of this thread's conv1 outputs into gs (kTile x HIDP).
template <int C>
DMX_DEVICE void store_g(const float2 (&acc)[Dc<C>::PM][Dc<C>::HN / 2], const DConvArgs& a,
                        float mean, float inv, float* gs) {
  using S = Dc<C>;
  const int tid = threadIdx.x, hg = tid / S::PG, pg = tid % S::PG;
#pragma unroll
  for (int j = 0; j < S::HN; ++j) {
    const int h = hg * S::HN + j;
    const float scale = inv * a.n1w[h];
    const float shift = a.n1b[h] - mean * scale;
#pragma unroll
    for (int i = 0; i < S::PM; ++i) {
      const float y = (j & 1) ? acc[i][j / 2].y : acc[i][j / 2].x;
      gs[(pg + i * S::PG) * S::HIDP + h] = gelu(y * scale + shift);
    }
  }
  if (S::HIDP > S::HID)
    for (int p = tid; p < kTile; p += kThreads)
#pragma unroll
      for (int h = S::HID; h < S::HIDP; ++h) gs[p * S::HIDP + h] = 0.f;
}

// conv2 over the g rows of a tile: x[p][c] += gamma * GLU(GN2(z)).
template <int C>
DMX_DEVICE void conv2_out(const float* gs, int np, const DConvArgs& a, float* xt, float mean2,
                          float inv2) {
  using S = Dc<C>;
  const int c = threadIdx.x % C, g0 = threadIdx.x / C;
  float2 w[S::HID];  // (value, gate) weights of channel c
#pragma unroll
  for (int h = 0; h < S::HID; ++h)
    w[h] = *reinterpret_cast<const float2*>(a.w2 + (int64_t)h * a.w2_ld + 2 * c);
  const float2 bias = *reinterpret_cast<const float2*>(a.b2 + 2 * c);
  const float vs = inv2 * a.n2w[c];
  const float vsh = a.n2b[c] - mean2 * vs;
  const float gsc = inv2 * a.n2w[c + C];
  const float gsh = a.n2b[c + C] - mean2 * gsc;
  const float gamma = a.gamma[c];
  for (int p = g0; p < np; p += S::G) {
    const float* gp = gs + p * S::HIDP;
    float2 z = bias;
#pragma unroll
    for (int h = 0; h < S::HIDP; h += 4) {
      const float4 g4 = *reinterpret_cast<const float4*>(gp + h);
      z = __ffma2_rn(w[h], make_float2(g4.x, g4.x), z);
      if (h + 1 < S::HID) z = __ffma2_rn(w[h + 1], make_float2(g4.y, g4.y), z);
      if (h + 2 < S::HID) z = __ffma2_rn(w[h + 2], make_float2(g4.z, g4.z), z);
      if (h + 3 < S::HID) z = __ffma2_rn(w[h + 3], make_float2(g4.w, g4.w), z);
    }
    const float value = z.x * vs + vsh;
    const float gate = z.y * gsc + gsh;
    float* o = xt + (int64_t)p * C + c;
    const float r = *o + gamma * (value * sigmoid(gate));
    *o = a.round_out ? round_tf32(r) : r;
  }
}

// Moments of z = conv2(g) over the tile's positions p < np without forming z:
// with g~ = (g, 1) and w~_n = (conv2 column n, its bias), sum_n z_n = v.g~ and
// sum_n z_n^2 = g~'Mg~ (v, M from the host: zq holds v, then M row by row at a
// stride of ZL floats, staged in shared memory). One position per thread and
// pass, f32 per position, f64 across them.
template <int C>
struct Zq {
  static constexpr int ACT = C / 8 + 1;
  static constexpr int ZL = (ACT + 3) / 4 * 4;
  static constexpr int N = ZL * (ACT + 1);
};

template <int C>
DMX_DEVICE void z_moments(const float* gs, int np, const float* zq, double& s, double& q) {
  using S = Dc<C>;
  using Z = Zq<C>;
  s = 0.0;
  q = 0.0;
  for (int p = threadIdx.x; p < np; p += kThreads) {
    const float* gp = gs + p * S::HIDP;
    float g[Z::ZL];
#pragma unroll
    for (int j = 0; j < Z::ZL; ++j) g[j] = j < S::HID ? gp[j] : (j == S::HID ? 1.0f : 0.f);
    float l = 0.f;
#pragma unroll
    for (int j = 0; j < Z::ZL; ++j) l = fmaf(zq[j], g[j], l);
    float qf = 0.f;
#pragma unroll 1
    for (int i = 0; i < Z::ACT; ++i) {
      const float4* mr = reinterpret_cast<const float4*>(zq + Z::ZL * (1 + i));
      float t = 0.f;
#pragma unroll
      for (int j4 = 0; j4 < Z::ZL / 4; ++j4) {
        const float4 m = mr[j4];
        t = fmaf(m.x, g[4 * j4], t);
        t = fmaf(m.y, g[4 * j4 + 1], t);
        t = fmaf(m.z, g[4 * j4 + 2], t);
        t = fmaf(m.w, g[4 * j4 + 3], t);
      }
      qf = fmaf(i < S::HID ? gp[i] : 1.0f, t, qf);
    }
    s += (double)l;
    q += (double)qf;
  }
}

template <int C>
DMX_DEVICE void stage_zq(const float* zq, float* zqs) {
  for (int i = threadIdx.x; i < Zq<C>::N; i += kThreads) zqs[i] = zq[i];
}

// Row moments of z for the tensor-core DConv path (three GEMMs, runtime.cu):
// y (positions, ld) is conv1's output with its row moments in st1 (sum, sum
// of squares); per position g = GELU(GroupNorm1(y)) and the quadratic form
// above; per CTA one f64 partial per row, part[row][blockIdx.x], added in
// order afterwards (stats.cu), so the moments do not depend on scheduling or
// on the other rows of the launch. Grid (ceil(T / 256), rows). Each thread keeps its g~ in
// its own column of shared memory for the rolled loop over M's rows.
template <int C>
__global__ void __launch_bounds__(256) dconv_zstats_kernel(const float* y, int ld, int T,
                                                           const float* n1w, const float* n1b,
                                                           const double* st1, double* part,
                                                           const float* zq) {
  using Z = Zq<C>;
  constexpr int HID = C / 8;
  extern __shared__ __align__(16) float zsm[];
  float* zqs = zsm;              // Z::N
  float* gcol = zsm + Z::N;      // [ZL][256]
  __shared__ float sc[HID], sh[HID];
  __shared__ double red[16];
  const int row = blockIdx.y, tid = threadIdx.x;
  for (int i = tid; i < Z::N; i += 256) zqs[i] = zq[i];
  if (tid < HID) {
    const double cnt = (double)HID * T;
    const double m = st1[2 * row] / cnt;
    const double var = fmax(st1[2 * row + 1] / cnt - m * m, 0.0);
    const float inv = 1.0f / sqrtf((float)(var + 1e-5));
    sc[tid] = inv * n1w[tid];
    sh[tid] = n1b[tid] - (float)m * sc[tid];
  }
  __syncthreads();
  const int t = blockIdx.x * 256 + tid;
  float l = 0.f, qf = 0.f;
  if (t < T) {
    const float* yp = y + ((int64_t)row * T + t) * ld;
    float g[Z::ZL];
#pragma unroll
    for (int j = 0; j < Z::ZL; ++j) {
      g[j] = j < HID ? gelu(yp[j] * sc[j] + sh[j]) : (j == HID ? 1.0f : 0.f);
      gcol[j * 256 + tid] = g[j];
      l = fmaf(zqs[j], g[j], l);
    }
#pragma unroll 1
    for (int i = 0; i < Z::ACT; ++i) {
      const float4* mr = reinterpret_cast<const float4*>(zqs + Z::ZL * (1 + i));
      float tt = 0.f;
#pragma unroll
      for (int j4 = 0; j4 < Z::ZL / 4; ++j4) {
        const float4 m = mr[j4];
        tt = fmaf(m.x, g[4 * j4], tt);
        tt = fmaf(m.y, g[4 * j4 + 1], tt);
        tt = fmaf(m.z, g[4 * j4 + 2], tt);
        tt = fmaf(m.w, g[4 * j4 + 3], tt);
      }
      qf = fmaf(gcol[i * 256 + tid], tt, qf);
    }
  }
  double ds = l, dq = qf;
  warp_sum2(ds, dq);
  if ((tid & 31) == 0) {
    red[2 * (tid >> 5)] = ds;
    red[2 * (tid >> 5) + 1] = dq;
  }
  __syncthreads();
  if (tid == 0) {
    double a0 = 0.0, a1 = 0.0;
    for (int w = 0; w < 8; ++w) {
      a0 += red[2 * w];
      a1 += red[2 * w + 1];
    }
    double* e = part + ((int64_t)row * gridDim.x + blockIdx.x) * 2;
    e[0] = a0;
    e[1] = a1;
  }
}

template <int C>
struct Smem {
  using S = Dc<C>;
  static constexpr size_t kRow = sizeof(float) * (S::XS + S::WS + S::YS);
  static constexpr size_t kConv1 = sizeof(float) * (S::XS + S::WS);
  static constexpr size_t kConv2 = sizeof(float) * S::YS;
};

// One CTA per row of T <= kTile positions: the whole DConv layer.
template <int C>
__global__ void __launch_bounds__(kThreads, C >= 384 ? 1 : 2) dconv_row_kernel(const DConvArgs a) {
  using S = Dc<C>;
  extern __shared__ __align__(16) float smem[];
  float* xs = smem;
  float* ws = xs + S::XS;
  float* gs = ws + S::WS;
  __shared__ double red[2 * kWarps];
  __shared__ __align__(16) float zqs[Zq<C>::N];
  const int row = blockIdx.x, T = a.T;
  float* xr = a.x + (int64_t)row * T * C;
  stage_zq<C>(a.zq_dev, zqs);

  float2 acc[S::PM][S::HN / 2];
  conv1_tile<C>(xr, T, 0, a.dil, a, xs, ws, acc);
  double s, q;
  conv1_moments<C>(acc, T, s, q);
  block_sum2(s, q, red);
  float mean, inv;
  moments_to_norm(s, q, (double)S::HID * T, mean, inv);
  store_g<C>(acc, a, mean, inv, gs);
  __syncthreads();

  z_moments<C>(gs, T, zqs, s, q);
  block_sum2(s, q, red);
  float mean2, inv2;
  moments_to_norm(s, q, 2.0 * C * T, mean2, inv2);
  conv2_out<C>(gs, T, a, xr, mean2, inv2);
}

// Tiled, step 1: conv1 of one tile -> y (HBM, compact HID channels) and the
// tile's moments.
template <int C>
__global__ void __launch_bounds__(kThreads, C >= 384 ? 1 : 2) dconv_conv1_kernel(const DConvArgs a) {
  using S = Dc<C>;
  extern __shared__ __align__(16) float smem[];
  float* xs = smem;
  float* ws = xs + S::XS;
  __shared__ double red[2 * kWarps];
  const int tile = blockIdx.x, row = blockIdx.y, T = a.T;
  const int t0 = tile * kTile, np = min(kTile, T - t0);
  const float* xr = a.x + (int64_t)row * T * C;

  float2 acc[S::PM][S::HN / 2];
  conv1_tile<C>(xr, T, t0, a.dil, a, xs, ws, acc);
  double s, q;
  conv1_moments<C>(acc, np, s, q);
  block_sum2(s, q, red);
  if (threadIdx.x == 0) {
    double* part = a.part1 + 2 * ((int64_t)row * a.tiles + tile);
    part[0] = s;
    part[1] = q;
  }
  const int hg = threadIdx.x / S::PG, pg = threadIdx.x % S::PG;
  float* yr = a.y + ((int64_t)row * T + t0) * S::HID;
#pragma unroll
  for (int i = 0; i < S::PM; ++i) {
    const int p = pg + i * S::PG;
    if (p < np)
#pragma unroll
      for (int j = 0; j < S::HN / 2; ++j)
        *reinterpret_cast<float2*>(yr + (int64_t)p * S::HID + hg * S::HN + 2 * j) = acc[i][j];
  }
}

// Tiled, steps 2 (OUT = false: z moments per tile) and 3 (OUT = true: the
// residual update).
template <int C, bool OUT>
__global__ void __launch_bounds__(kThreads, C >= 384 ? 1 : 2) dconv_conv2_kernel(const DConvArgs a) {
  using S = Dc<C>;
  extern __shared__ __align__(16) float smem[];
  float* gs = smem;
  __shared__ double red[2 * kWarps];
  __shared__ __align__(16) float zqs[OUT ? 4 : Zq<C>::N];
  const int tile = blockIdx.x, row = blockIdx.y, T = a.T;
  const int t0 = tile * kTile, np = min(kTile, T - t0);
  if (!OUT) stage_zq<C>(a.zq_dev, zqs);

  float mean, inv;
  row_moments(a.part1 + 2 * (int64_t)row * a.tiles, a.tiles, (double)S::HID * T, mean, inv, red);
  const float* yr = a.y + ((int64_t)row * T + t0) * S::HID;
  for (int i = threadIdx.x; i < kTile * S::HIDP; i += kThreads) {
    const int p = i / S::HIDP, h = i - p * S::HIDP;
    float g = 0.f;
    if (p < np && h < S::HID) {
      const float scale = inv * a.n1w[h];
      const float shift = a.n1b[h] - mean * scale;
      g = gelu(yr[(int64_t)p * S::HID + h] * scale + shift);
    }
    gs[i] = g;
  }
  float mean2 = 0.f, inv2 = 0.f;
  if (OUT) {
    __syncthreads();  // red reused
    row_moments(a.part2 + 2 * (int64_t)row * a.tiles, a.tiles, 2.0 * C * T, mean2, inv2, red + 2);
  }
  __syncthreads();
  double s, q;
  float* xt = a.x + ((int64_t)row * T + t0) * C;
  if (OUT)
    conv2_out<C>(gs, np, a, xt, mean2, inv2);
  else
    z_moments<C>(gs, np, zqs, s, q);
  if (!OUT) {
    block_sum2(s, q, red);
    if (threadIdx.x == 0) {
      double* part = a.part2 + 2 * ((int64_t)row * a.tiles + tile);
      part[0] = s;
      part[1] = q;
    }
  }
}

template <class K>
void set_smem(K kernel, size_t bytes) {
  if (bytes > 48 * 1024)
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

template <int C>
void launch_c(const DConvArgs& a, cudaStream_t s) {
  using M = Smem<C>;
  static PerDevice configured;
  if (configured.first()) {
    set_smem(dconv_row_kernel<C>, M::kRow);
    set_smem(dconv_conv1_kernel<C>, M::kConv1);
    set_smem(dconv_conv2_kernel<C, false>, M::kConv2);
    set_smem(dconv_conv2_kernel<C, true>, M::kConv2);
  }
  if (a.T <= kTile) {
    dconv_row_kernel<C><<<a.rows, kThreads, M::kRow, s>>>(a);
    return;
  }
  const dim3 grid(a.tiles, a.rows);
  dconv_conv1_kernel<C><<<grid, kThreads, M::kConv1, s>>>(a);
  dconv_conv2_kernel<C, false><<<grid, kThreads, M::kConv2, s>>>(a);
  dconv_conv2_kernel<C, true><<<grid, kThreads, M::kConv2, s>>>(a);
}

template <int C>
void launch_zstats_c(const float* y, int ld, int rows, int T, const float* n1w, const float* n1b,
                     const double* st1, double* st2, double* part, const float* zq,
                     cudaStream_t s) {
  const size_t bytes = sizeof(float) * (Zq<C>::N + Zq<C>::ZL * 256);
  static PerDevice configured;
  if (configured.first()) set_smem(dconv_zstats_kernel<C>, bytes);
  dconv_zstats_kernel<C><<<dim3(dconv_zstats_parts(T), rows), 256, bytes, s>>>(y, ld, T, n1w, n1b,
                                                                              st1, part, zq);
  launch_sum_partials(part, dconv_zstats_parts(T), rows, st2, s);
}

}  // namespace

int dconv_zstats_parts(int T) { return (T + 255) / 256; }

bool launch_dconv_zstats(int C, const float* y, int ld, int rows, int T, const float* n1w,
                         const float* n1b, const double* st1, double* st2, double* part,
                         const float* zq, cudaStream_t s) {
  if (!zq || !part || rows <= 0 || T <= 0 || ld < C / 8) return false;
  switch (C) {
    case 192: launch_zstats_c<192>(y, ld, rows, T, n1w, n1b, st1, st2, part, zq, s); return true;
    case 384: launch_zstats_c<384>(y, ld, rows, T, n1w, n1b, st1, st2, part, zq, s); return true;
    default: return false;
  }
}

int dconv_tiles(int T) { return (T + kTile - 1) / kTile; }

bool dconv_row_fused(int T) { return T <= kTile; }

bool launch_dconv(const DConvArgs& a, cudaStream_t s) {
  if (a.dil < 1 || a.dil > kMaxDil || a.rows <= 0 || a.T <= 0 || !a.zq_dev) return false;
  if (a.T > kTile && (!a.y || !a.part1 || !a.part2 || a.tiles != dconv_tiles(a.T))) return false;
  switch (a.C) {
    case 48: launch_c<48>(a, s); return true;
    case 96: launch_c<96>(a, s); return true;
    case 192: launch_c<192>(a, s); return true;
    case 384: launch_c<384>(a, s); return true;
    default: return false;
  }
}

}  // namespace dmx
