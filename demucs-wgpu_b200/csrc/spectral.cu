// Spectrogram front and back end, memory-bound kernels:
//  * stft_cac: reflect pad (spec.rs:62-113, 204-236) + periodic Hann +
//    4096-point FFT + 1/64 normalisation + CaC packing (spec.rs:240-254),
//    written channels-last (b, f, t, 4), with the per-segment moments of the
//    packed spectrogram accumulated in f64 on the way out (host.rs:523-543).
//  * wave_moments: per-segment moments of the waveform.
//  * norm_finalize: mean / unbiased std / 1/(1e-5+std) per segment.
//  * istft_frames + istft_ola: denormalise (host.rs:466-469), unpack
//    (spec.rs:268-300), zero Nyquist bin and border frames (spec.rs:312-340),
//    inverse FFT x window x 1/64, overlap-add divided by the window-squared
//    envelope, crop (stft.rs:204-295, spec.rs:117-175), plus the denormalised
//    time branch (host.rs:499-512) into (b, source, channel, sample).
#include "common.cuh"
#include "kernels.h"

namespace dmx {

namespace {

// Radix-2 decimation-in-time FFT of 4096 complex values in shared memory.
// `sign` = -1 forward, +1 inverse; tw[k] = exp(-2 pi i k / 4096), k < 2048.
DMX_DEVICE void fft4096(float* re, float* im, const float2* __restrict__ tw, float sign) {
  for (int h = 1; h < kNfft; h <<= 1) {
    const int step = kNfft / (2 * h);
    for (int j = threadIdx.x; j < kNfft / 2; j += blockDim.x) {
      const int k = j % h;
      const int a = (j / h) * 2 * h + k;
      const int b = a + h;
      const float2 w = tw[k * step];
      const float wr = w.x, wi = sign * -w.y;  // exp(sign * 2 pi i k / len)
      const float xr = re[b] * wr - im[b] * wi;
      const float xi = re[b] * wi + im[b] * wr;
      re[b] = re[a] - xr;
      im[b] = im[a] - xi;
      re[a] += xr;
      im[a] += xi;
    }
    __syncthreads();
  }
}

DMX_DEVICE int bitrev12(int n) { return __brev(n) >> 20; }

__global__ void __launch_bounds__(512) stft_cac_kernel(const float* __restrict__ mix,
                                                       const float* __restrict__ window,
                                                       const float2* __restrict__ tw,
                                                       float* __restrict__ out,
                                                       double* __restrict__ stats) {
  __shared__ float re[kNfft], im[kNfft];
  __shared__ double red[2][16];
  const int t = blockIdx.x, b = blockIdx.y;
  const float* x0 = mix + (int64_t)b * 2 * kSegment;
  const float* x1 = x0 + kSegment;
  for (int n = threadIdx.x; n < kNfft; n += blockDim.x) {
    // kept frame t is torch frame t+2; its samples are the pad1d output
    // [1024 t, 1024 t + 4096), i.e. mix index 1024 t + n - 1536 reflected.
    int idx = t * kHop + n - kPad;
    if (idx < 0) idx = -idx;
    if (idx >= kSegment) idx = 2 * (kSegment - 1) - idx;
    const float w = window[n];
    const int r = bitrev12(n);
    re[r] = x0[idx] * w;
    im[r] = x1[idx] * w;
  }
  __syncthreads();
  fft4096(re, im, tw, -1.f);
  double s = 0.0, q = 0.0;
  const float norm = 1.0f / 64.0f;
  for (int k = threadIdx.x; k < kBins; k += blockDim.x) {
    const int nk = (kNfft - k) & (kNfft - 1);
    const float zr = re[k], zi = im[k], cr = re[nk], ci = im[nk];
    float4 v;
    v.x = 0.5f * (zr + cr) * norm;
    v.y = 0.5f * (zi - ci) * norm;
    v.z = 0.5f * (zi + ci) * norm;
    v.w = -0.5f * (zr - cr) * norm;
    *reinterpret_cast<float4*>(out + (((int64_t)b * kBins + k) * kFrames + t) * 4) = v;
    s += (double)v.x + (double)v.y + (double)v.z + (double)v.w;
    q += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
  }
  s = warp_sum(s);
  q = warp_sum(q);
  if ((threadIdx.x & 31) == 0) {
    red[0][threadIdx.x / 32] = s;
    red[1][threadIdx.x / 32] = q;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int nw = blockDim.x / 32;
    s = threadIdx.x < nw ? red[0][threadIdx.x] : 0.0;
    q = threadIdx.x < nw ? red[1][threadIdx.x] : 0.0;
    s = warp_sum(s);
    q = warp_sum(q);
    if (threadIdx.x == 0) {
      atomicAdd(&stats[2 * b], s);
      atomicAdd(&stats[2 * b + 1], q);
    }
  }
}

__global__ void wave_moments_kernel(const float* __restrict__ mix, int64_t n,
                                    double* __restrict__ stats) {
  __shared__ double red[2][32];
  const int b = blockIdx.y;
  const float* x = mix + (int64_t)b * n;
  double s = 0.0, q = 0.0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const double v = x[i];
    s += v;
    q += v * v;
  }
  s = warp_sum(s);
  q = warp_sum(q);
  if ((threadIdx.x & 31) == 0) {
    red[0][threadIdx.x / 32] = s;
    red[1][threadIdx.x / 32] = q;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int nw = blockDim.x / 32;
    s = threadIdx.x < nw ? red[0][threadIdx.x] : 0.0;
    q = threadIdx.x < nw ? red[1][threadIdx.x] : 0.0;
    s = warp_sum(s);
    q = warp_sum(q);
    if (threadIdx.x == 0) {
      atomicAdd(&stats[2 * b], s);
      atomicAdd(&stats[2 * b + 1], q);
    }
  }
}

// norm[b] = {mean, 1/(1e-5 + std), std, -mean/std} (host.rs:250-261, 466-469;
// ops.rs:1494-1509, 1585-1590).
__global__ void norm_finalize_kernel(const double* __restrict__ stats, double count, int B,
                                     float4* __restrict__ norm) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const double sum = stats[2 * b], sq = stats[2 * b + 1];
  const double mean = sum / count;
  const double var = fmax((sq - sum * sum / count) / (count - 1.0), 0.0);
  const float meanf = (float)mean;
  const float sd = (float)sqrt(var);
  float4 r;
  r.x = meanf;
  r.y = 1.0f / (1e-5f + sd);
  r.z = sd;
  r.w = -meanf / sd;
  norm[b] = r;
}

// One CTA per (b, source, frame t): both audio channels of the source in one
// complex inverse FFT (z = A + iB for Hermitian A, B gives a + ib).
__global__ void __launch_bounds__(512) istft_frames_kernel(const float* __restrict__ spec,
                                                           const float4* __restrict__ norm,
                                                           const float* __restrict__ window,
                                                           const float2* __restrict__ tw,
                                                           float* __restrict__ frames) {
  __shared__ float re[kNfft], im[kNfft];
  const int t = blockIdx.x, s = blockIdx.y, b = blockIdx.z;
  const float4 nz = norm[b];
  const float o2 = nz.w, sd = nz.z;
  // spec (b, f, t, 16): channel s*4 + a*2 + {re, im}
  for (int k = threadIdx.x; k < kNfft; k += blockDim.x) {
    float zr = 0.f, zi = 0.f;
    if (k < kBins) {
      const float4 v = *reinterpret_cast<const float4*>(
          spec + (((int64_t)b * kBins + k) * kFrames + t) * 16 + s * 4);
      const float ar = (v.x - o2) * sd, ai = (v.y - o2) * sd;
      const float br = (v.z - o2) * sd, bi = (v.w - o2) * sd;
      if (k == 0) {  // irfft ignores the imaginary part of the DC bin
        zr = ar;
        zi = br;
      } else {
        zr = ar - bi;
        zi = ai + br;
      }
    } else if (k > kBins) {
      const int m = kNfft - k;  // Z[N-m] = conj(A[m]) + i conj(B[m])
      const float4 v = *reinterpret_cast<const float4*>(
          spec + (((int64_t)b * kBins + m) * kFrames + t) * 16 + s * 4);
      const float ar = (v.x - o2) * sd, ai = (v.y - o2) * sd;
      const float br = (v.z - o2) * sd, bi = (v.w - o2) * sd;
      zr = ar + bi;
      zi = -ai + br;
    }  // k == 2048: the zero Nyquist bin
    const int r = bitrev12(k);
    re[r] = zr;
    im[r] = zi;
  }
  __syncthreads();
  fft4096(re, im, tw, +1.f);
  const float inv_n = 64.0f / 4096.0f;
  float* fa = frames + ((((int64_t)b * 4 + s) * 2 + 0) * kFrames + t) * kNfft;
  float* fb = frames + ((((int64_t)b * 4 + s) * 2 + 1) * kFrames + t) * kNfft;
  for (int n = threadIdx.x; n < kNfft; n += blockDim.x) {
    const float w = window[n];
    fa[n] = re[n] * inv_n * w;
    fb[n] = im[n] * inv_n * w;
  }
}

// out (b, s, a, j) = time(b, j, s*2+a) denormalised + sum_f frames / env.
__global__ void istft_ola_kernel(const float* __restrict__ frames,
                                 const float* __restrict__ envelope,  // [1024]
                                 const float* __restrict__ time_branch,  // (b, L, 8)
                                 const float4* __restrict__ norm_t, float* __restrict__ out,
                                 int B) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int b = blockIdx.y;
  if (j >= kSegment) return;
  const int64_t i = j + kPad + kNfft / 2;  // index in the centred istft signal
  const int fhi = (int)(i / kHop);
  const float env = envelope[i % kHop];
  const float4 nt = norm_t[b];
  const float4 t0 = *reinterpret_cast<const float4*>(time_branch + ((int64_t)b * kSegment + j) * 8);
  const float4 t1 = *reinterpret_cast<const float4*>(time_branch + ((int64_t)b * kSegment + j) * 8 + 4);
  const float tv[8] = {t0.x, t0.y, t0.z, t0.w, t1.x, t1.y, t1.z, t1.w};
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const float* fr = frames + ((int64_t)b * 8 + r) * kFrames * kNfft;
    float y = 0.f;
#pragma unroll
    for (int f = fhi - 3; f <= fhi; ++f) {
      const int t = f - 2;
      if (t >= 0 && t < kFrames) y += fr[(int64_t)t * kNfft + (i - (int64_t)f * kHop)];
      else y += 0.f;
    }
    const float wave = y / env;
    const float time = (tv[r] - nt.w) * nt.z;
    out[((int64_t)b * 8 + r) * kSegment + j] = time + wave;
  }
}

}  // namespace

void launch_stft_cac(const float* mix, int B, const float* window, const float2* tw, float* out,
                     double* stats, cudaStream_t s) {
  stft_cac_kernel<<<dim3(kFrames, B), 512, 0, s>>>(mix, window, tw, out, stats);
}

void launch_wave_moments(const float* mix, int B, int64_t n, double* stats, cudaStream_t s) {
  wave_moments_kernel<<<dim3(148, B), 512, 0, s>>>(mix, n, stats);
}

void launch_norm_finalize(const double* stats, double count, int B, float4* norm,
                          cudaStream_t s) {
  norm_finalize_kernel<<<(B + 63) / 64, 64, 0, s>>>(stats, count, B, norm);
}

void launch_istft(const float* spec, const float4* norm, const float* window, const float2* tw,
                  float* frames, const float* envelope, const float* time_branch,
                  const float4* norm_t, float* out, int B, cudaStream_t s) {
  istft_frames_kernel<<<dim3(kFrames, 4, B), 512, 0, s>>>(spec, norm, window, tw, frames);
  istft_ola_kernel<<<dim3((kSegment + 255) / 256, B), 256, 0, s>>>(frames, envelope, time_branch,
                                                                  norm_t, out, B);
}

}  // namespace dmx
