// The first encoder convolutions of both branches (host.rs:577-622 and the
// time-branch twin): Cin = 4 (the CaC spectrogram) or 2 (the waveform), eight
// taps at stride 4 along one axis with padding 2, Cout = 48, the segment's
// normalisation applied on load and GELU on the way out.
//
// With K = 8 Cin <= 32 these are too thin for the tensor-core GEMM (a 16-byte
// A row) and the general SIMT GEMM spends its time on tile bookkeeping. Here
// one CTA takes 128 consecutive output positions: each thread gathers the K
// normalised inputs of one position into registers and accumulates 24 of the
// 48 channels; the weights (at most 6 KB) travel as a launch parameter, so the
// FMAs read them straight from the constant bank. The 128 x 48 output tile is
// staged in shared memory and leaves as one contiguous, coalesced 24 KB store.
// fp32 throughout.
#include "common.cuh"
#include "conv_gemm.cuh"

namespace dmx {

namespace {

constexpr int kCo = 48, kBM = 128, kRow = kCo + 4;  // padded staging row (conflict-free)

template <int CIN>
struct FirstConvW {
  float w[8 * CIN][kCo];
  float b[kCo];
};

// 24 channels from 24 h of one position, weights from the constant bank;
// channel pairs on the paired fp32 FMA (each lane rounds as fmaf does)
template <int CIN, int H>
DMX_DEVICE void accumulate(const FirstConvW<CIN>& cw, const float* in, float* acc) {
  float2 a2[12];
#pragma unroll
  for (int j = 0; j < 12; ++j) a2[j] = make_float2(cw.b[24 * H + 2 * j], cw.b[24 * H + 2 * j + 1]);
#pragma unroll
  for (int k = 0; k < 8 * CIN; ++k) {
    const float2 xk = make_float2(in[k], in[k]);
#pragma unroll
    for (int j = 0; j < 12; ++j)
      a2[j] = __ffma2_rn(xk, make_float2(cw.w[k][24 * H + 2 * j], cw.w[k][24 * H + 2 * j + 1]), a2[j]);
  }
#pragma unroll
  for (int j = 0; j < 12; ++j) {
    acc[2 * j] = a2[j].x;
    acc[2 * j + 1] = a2[j].y;
  }
}

template <int CIN>
__global__ void __launch_bounds__(256) first_conv_kernel(const ConvParams p,
                                                         const __grid_constant__ FirstConvW<CIN> cw) {
  constexpr int K = 8 * CIN;
  __shared__ __align__(16) float os[kBM * kRow];
  const int tid = threadIdx.x;

  const int64_t M = (int64_t)p.B * p.Hq * p.Wq;
  const int64_t m0 = (int64_t)blockIdx.x * kBM;
  const int pl = tid % kBM, half = tid / kBM;  // position, channels 24 half .. +24
  const int64_t pos = m0 + pl;
  float in[K];
  if (pos < M) {
    const int64_t plane = (int64_t)p.Hq * p.Wq;
    const int b = (int)(pos / plane);
    const int64_t rem = pos - (int64_t)b * plane;
    const int y = (int)(rem / p.Wq), x = (int)(rem % p.Wq);
    const float4 nz = reinterpret_cast<const float4*>(p.pro_scale)[b];
    const float* xb = p.x + (int64_t)b * p.i_bs;
#pragma unroll
    for (int tap = 0; tap < 8; ++tap) {
      const int iy = y * p.sy + p.dy[tap], ix = x * p.sx + p.dx[tap];
      const bool inside = iy >= 0 && iy < p.Hin && ix >= 0 && ix < p.Win;
      const float* src = xb + (int64_t)iy * p.i_ys + (int64_t)ix * p.i_xs;
#pragma unroll
      for (int ci = 0; ci < CIN; ++ci)
        in[tap * CIN + ci] = inside ? (__ldg(src + (int64_t)ci * p.i_cs) - nz.x) * nz.y : 0.f;
    }
  } else {
#pragma unroll
    for (int k = 0; k < K; ++k) in[k] = 0.f;
  }

  float acc[24];
  if (half == 0)  // warp-uniform
    accumulate<CIN, 0>(cw, in, acc);
  else
    accumulate<CIN, 1>(cw, in, acc);
  float4* orow = reinterpret_cast<float4*>(&os[pl * kRow + 24 * half]);
#pragma unroll
  for (int c = 0; c < 6; ++c)
    orow[c] = make_float4(gelu(acc[4 * c]), gelu(acc[4 * c + 1]), gelu(acc[4 * c + 2]),
                          gelu(acc[4 * c + 3]));
  __syncthreads();
  // the tile's positions are consecutive rows of the channels-last output
  const int rows = M - m0 < kBM ? (int)(M - m0) : kBM;
  float4* dst = reinterpret_cast<float4*>(p.out + m0 * kCo);
  for (int i = tid; i < rows * (kCo / 4); i += blockDim.x) {
    const int r = i / (kCo / 4), c = i % (kCo / 4);
    dst[i] = *reinterpret_cast<const float4*>(&os[r * kRow + 4 * c]);
  }
}

template <int CIN>
void launch_cin(const ConvParams& p, const float* w_host, unsigned grid, cudaStream_t s) {
  FirstConvW<CIN> cw;
  for (int k = 0; k < 8 * CIN; ++k)
    for (int n = 0; n < kCo; ++n) cw.w[k][n] = w_host[k * kCo + n];
  for (int n = 0; n < kCo; ++n) cw.b[n] = w_host[8 * CIN * kCo + n];
  first_conv_kernel<CIN><<<grid, 256, 0, s>>>(p, cw);
}

}  // namespace

bool launch_first_conv(const ConvParams& p, int pro, int epi, const float* w_host, cudaStream_t s) {
  if (pro != PRO_BATCH_AFFINE || epi != EPI_GELU || (p.Cin != 2 && p.Cin != 4) || p.ntaps != 8 ||
      p.K != 8 * p.Cin || p.N != kCo || p.Npad < kCo || p.epi_add || p.round_out || p.o_lim ||
      p.o_off != 0 || p.o_xs != kCo || p.o_ys != (int64_t)p.Wq * kCo ||
      p.o_bs != (int64_t)p.Hq * p.Wq * kCo || (reinterpret_cast<uintptr_t>(p.out) & 15))
    return false;
  const int64_t M = (int64_t)p.B * p.Hq * p.Wq;
  const unsigned grid = (unsigned)((M + kBM - 1) / kBM);
  if (p.Cin == 4)
    launch_cin<4>(p, w_host, grid, s);
  else
    launch_cin<2>(p, w_host, grid, s);
  return true;
}

}  // namespace dmx
