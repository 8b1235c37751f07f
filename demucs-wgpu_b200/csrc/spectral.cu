// Spectrogram front and back end, memory-bound kernels:
//  * stft_cac: reflect pad (spec.rs:62-113, 204-236) + periodic Hann +
//    4096-point FFT + 1/64 normalisation + CaC packing (spec.rs:240-254),
//    written channels-last (b, f, t, 4), with the per-segment moments of the
//    packed spectrogram formed in f64 on the way out (host.rs:523-543): one
//    partial per (segment, frame).
//  * wave_moments: per-segment moments of the waveform, one partial per
//    (segment, block of a fixed grid).
//  * norm_finalize: adds a segment's partials in order, then mean / unbiased
//    std / 1/(1e-5+std). No atomics: a segment's moments do not depend on the
//    other segments of the batch or on scheduling.
//  * istft: denormalise (host.rs:466-469), unpack (spec.rs:268-300), zero
//    Nyquist bin and border frames (spec.rs:312-340), inverse FFT x window x
//    1/64, overlap-add divided by the window-squared envelope, crop
//    (stft.rs:204-295, spec.rs:117-175), plus the denormalised time branch
//    (host.rs:499-512) into (b, source, channel, sample), in one kernel.
#include "common.cuh"
#include "kernels.h"

namespace dmx {

namespace {

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
      stats[((int64_t)b * gridDim.x + blockIdx.x) * 2] = s;
      stats[((int64_t)b * gridDim.x + blockIdx.x) * 2 + 1] = q;
    }
  }
}

// norm[b] = {mean, 1/(1e-5 + std), std, -mean/std} (host.rs:250-261, 466-469;
// ops.rs:1494-1509, 1585-1590).
__global__ void norm_finalize_kernel(const double* __restrict__ part, int nparts, double count,
                                     int B, float4* __restrict__ norm) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  double sum = 0.0, sq = 0.0;
  const double* e = part + (int64_t)b * nparts * 2;
  for (int k = 0; k < nparts; ++k) {
    sum += e[2 * k];
    sq += e[2 * k + 1];
  }
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

// ---------------------------------------------------------------------------
// iSTFT + overlap-add + time-branch sum, fused. One CTA per (source, 8 output
// hops, segment): it inverts the 11 frames that overlap its hops
// (both audio channels of the source in one complex inverse FFT, z = A + iB
// for Hermitian A, B gives a + ib), windows them and overlap-adds them in
// shared memory, then writes time + ola / envelope for its 8192 samples.
// No frame buffer touches HBM; the 3 frames shared with each neighbouring CTA
// are inverted twice.
//
// The 4096-point inverse FFT is 16 x 256 with 256 = 16 x 16: three passes of
// 16-point DFTs held in registers (256 threads, one DFT each), with the
// inter-pass twiddles between them; the work buffer's row stride (273) keeps
// the passes' shared-memory accesses (nearly) conflict-free.
constexpr int kIstftHops = 8;
constexpr int kIstftThreads = 256;
constexpr int kRow = 273;  // stride between the 16 rows of the FFT work buffer
constexpr size_t kIstftSmem = sizeof(float) * (2 * 16 * kRow + 2 * kIstftHops * kHop);

struct cpx {
  float x, y;
};
DMX_DEVICE cpx cmul(cpx a, cpx b) { return {a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x}; }

// inverse 4-point DFT in place: y_k = sum_n a_n i^(n k)
DMX_DEVICE void idft4(cpx& a0, cpx& a1, cpx& a2, cpx& a3) {
  const cpx s02 = {a0.x + a2.x, a0.y + a2.y}, d02 = {a0.x - a2.x, a0.y - a2.y};
  const cpx s13 = {a1.x + a3.x, a1.y + a3.y}, d13 = {a1.x - a3.x, a1.y - a3.y};
  a0 = {s02.x + s13.x, s02.y + s13.y};
  a2 = {s02.x - s13.x, s02.y - s13.y};
  a1 = {d02.x - d13.y, d02.y + d13.x};  // d02 + i d13
  a3 = {d02.x + d13.y, d02.y - d13.x};  // d02 - i d13
}

// inverse 16-point DFT of v (input in natural order) as 4 x 4; output k is
// left at v[4 (k % 4) + k / 4].
DMX_DEVICE void idft16(cpx (&v)[16]) {
  // e^(+2 pi i m / 16) for the products b*c of the twiddle step
  constexpr float c1 = 0.92387953251128674f, s1 = 0.38268343236508977f;
  constexpr float r2 = 0.70710678118654752f;
#pragma unroll
  for (int b = 0; b < 4; ++b) idft4(v[b], v[4 + b], v[8 + b], v[12 + b]);
  v[5] = cmul(v[5], {c1, s1});     // b*c = 1
  v[9] = cmul(v[9], {r2, r2});     // 2
  v[13] = cmul(v[13], {s1, c1});   // 3
  v[6] = cmul(v[6], {r2, r2});     // 2
  v[10] = {-v[10].y, v[10].x};     // 4: times i
  v[14] = cmul(v[14], {-r2, r2});  // 6
  v[7] = cmul(v[7], {s1, c1});     // 3
  v[11] = cmul(v[11], {-r2, r2});  // 6
  v[15] = cmul(v[15], {-c1, -s1}); // 9
#pragma unroll
  for (int c = 0; c < 4; ++c) idft4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
}
DMX_DEVICE int idft16_slot(int k) { return 4 * (k & 3) + (k >> 2); }

// e^(+2 pi i j / 4096), j < 4096, from the forward table tw[k] = e^(-2 pi i k / 4096)
DMX_DEVICE cpx w_inv(const float2* __restrict__ tw, int j) {
  const float2 t = __ldg(tw + (j & 2047));
  return j < 2048 ? cpx{t.x, -t.y} : cpx{-t.x, t.y};
}

// W^k for k = 0..15 from W^1, W^2, W^4, W^8 (at most three products deep,
// so the error stays within a few roundings of the table's).
DMX_DEVICE void powers16(cpx w1, cpx w2, cpx w4, cpx w8, cpx (&p)[16]) {
  p[0] = {1.f, 0.f};
  p[1] = w1;
  p[2] = w2;
  p[3] = cmul(w1, w2);
  p[4] = w4;
  p[5] = cmul(w1, w4);
  p[6] = cmul(w2, w4);
  p[7] = cmul(p[3], w4);
#pragma unroll
  for (int k = 0; k < 8; ++k) p[8 + k] = k == 0 ? w8 : cmul(p[k], w8);
}

// STFT of one frame per CTA (both audio channels in one complex FFT,
// z = x0 + i x1), 256 threads. The forward 4096-point FFT is taken as the
// conjugate of the inverse one of conj(z), with the same three radix-16
// register passes and twiddles as the iSTFT below; X lands in the work
// buffer in natural order for the CaC unpack (A[k] = (Z[k] + conj Z[N-k])/2,
// B[k] = (Z[k] - conj Z[N-k])/2i), written channels-last (b, f, t, 4) with the
// segment's moments summed in f64.
__global__ void __launch_bounds__(256) stft_cac_kernel(const float* __restrict__ mix,
                                                       const float* __restrict__ window,
                                                       const float2* __restrict__ tw,
                                                       float* __restrict__ out,
                                                       double* __restrict__ stats) {
  __shared__ float bre[16 * kRow], bim[16 * kRow];
  __shared__ double red[2][8];
  const int t = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
  const float* x0 = mix + (int64_t)b * 2 * kSegment;
  const float* x1 = x0 + kSegment;
  cpx v[16];
  // pass 1: thread m = tid, conj z[256 n2 + m]; kept frame t is torch frame
  // t + 2, whose samples are the reflect-padded mix at 1024 t + n - 1536
#pragma unroll
  for (int n2 = 0; n2 < 16; ++n2) {
    const int n = 256 * n2 + tid;
    int idx = t * kHop + n - kPad;
    if (idx < 0) idx = -idx;
    if (idx >= kSegment) idx = 2 * (kSegment - 1) - idx;
    const float w = __ldg(window + n);
    v[n2] = {__ldg(x0 + idx) * w, -__ldg(x1 + idx) * w};
  }
  idft16(v);
  {
    cpx wk[16];
    powers16(w_inv(tw, tid), w_inv(tw, 2 * tid), w_inv(tw, 4 * tid), w_inv(tw, 8 * tid), wk);
#pragma unroll
    for (int k1 = 0; k1 < 16; ++k1) {
      const cpx y = k1 == 0 ? v[idft16_slot(0)] : cmul(v[idft16_slot(k1)], wk[k1]);
      bre[k1 * kRow + tid] = y.x;
      bim[k1 * kRow + tid] = y.y;
    }
  }
  __syncthreads();
  {
    // pass 2: thread (k1, c), the 256-point DFT over m = 16 a + c, first level
    const int k1 = tid >> 4, c = tid & 15;
#pragma unroll
    for (int a = 0; a < 16; ++a) v[a] = {bre[k1 * kRow + 16 * a + c], bim[k1 * kRow + 16 * a + c]};
    __syncthreads();
    idft16(v);
    cpx wk[16];
    powers16(w_inv(tw, 16 * c), w_inv(tw, 32 * c), w_inv(tw, 64 * c), w_inv(tw, 128 * c), wk);
#pragma unroll
    for (int d = 0; d < 16; ++d) {
      const cpx u = (d == 0 || c == 0) ? v[idft16_slot(d)] : cmul(v[idft16_slot(d)], wk[d]);
      bre[k1 * kRow + 17 * d + c] = u.x;
      bim[k1 * kRow + 17 * d + c] = u.y;
    }
  }
  __syncthreads();
  {
    // pass 3: thread (d, k1), second level: X[k1 + 16 d + 256 e], e = 0..15
    const int d = tid >> 4, k1 = tid & 15;
#pragma unroll
    for (int c = 0; c < 16; ++c) v[c] = {bre[k1 * kRow + 17 * d + c], bim[k1 * kRow + 17 * d + c]};
    idft16(v);
    __syncthreads();
#pragma unroll
    for (int e = 0; e < 16; ++e) {  // X = conj of the inverse transform of conj z
      const int k = k1 + 16 * d + 256 * e;
      bre[k] = v[idft16_slot(e)].x;
      bim[k] = -v[idft16_slot(e)].y;
    }
  }
  __syncthreads();
  double s = 0.0, q = 0.0;
  const float norm = 1.0f / 64.0f;
  for (int k = tid; k < kBins; k += 256) {
    const int nk = (kNfft - k) & (kNfft - 1);
    const float zr = bre[k], zi = bim[k], cr = bre[nk], ci = bim[nk];
    float4 o;
    o.x = 0.5f * (zr + cr) * norm;
    o.y = 0.5f * (zi - ci) * norm;
    o.z = 0.5f * (zi + ci) * norm;
    o.w = -0.5f * (zr - cr) * norm;
    *reinterpret_cast<float4*>(out + (((int64_t)b * kBins + k) * kFrames + t) * 4) = o;
    s += (double)o.x + (double)o.y + (double)o.z + (double)o.w;
    q += (double)o.x * o.x + (double)o.y * o.y + (double)o.z * o.z + (double)o.w * o.w;
  }
  s = warp_sum(s);
  q = warp_sum(q);
  if ((tid & 31) == 0) {
    red[0][tid / 32] = s;
    red[1][tid / 32] = q;
  }
  __syncthreads();
  if (tid < 32) {
    s = tid < 8 ? red[0][tid] : 0.0;
    q = tid < 8 ? red[1][tid] : 0.0;
    s = warp_sum(s);
    q = warp_sum(q);
    if (tid == 0) {
      stats[((int64_t)b * kFrames + t) * 2] = s;
      stats[((int64_t)b * kFrames + t) * 2 + 1] = q;
    }
  }
}

// spec: the decoder output frame-major, (b, t, f, 16) with channel
// source*4 + audio channel*2 + {re, im}.
__global__ void __launch_bounds__(kIstftThreads, 2)
    istft_kernel(const float* __restrict__ spec, const float4* __restrict__ norm,
                 const float* __restrict__ window, const float2* __restrict__ tw,
                 const float* __restrict__ envelope, const float* __restrict__ time_branch,
                 const float4* __restrict__ norm_t, float* __restrict__ out) {
  extern __shared__ float sm[];
  float* bre = sm;                  // FFT work buffer, 16 rows x kRow
  float* bim = sm + 16 * kRow;
  float* acc = sm + 32 * kRow;      // overlap-add, 2 channels x (8 x 1024)
  constexpr int AC = kIstftHops * kHop;
  // source fastest: the 4 CTAs of one hop group read the same spectrogram
  // sectors close together in time
  const int tid = threadIdx.x, s = blockIdx.x, b = blockIdx.z;
  const int H0 = 3 + blockIdx.y * kIstftHops;  // first hop: centred-signal index i / 1024
  const float4 nz = norm[b];
  const float o2 = nz.w, sd = nz.z;
  const float inv_n = 64.0f / 4096.0f;
  // kept frame t is torch frame f = t + 2 and covers hops f .. f + 3
  const int t_lo = max(0, H0 - 5), t_hi = min(kFrames - 1, H0 + kIstftHops - 3);

  {
    for (int i = tid; i < 2 * AC; i += kIstftThreads) acc[i] = 0.f;
    for (int t = t_lo; t <= t_hi; ++t) {
      // pass 1: thread m = tid, Z[256 n2 + m] for n2 = 0..15 straight from the
      // spectrogram; all 16 loads are issued before any is used
      cpx v[16];
      {
        const float* fr = spec + ((int64_t)b * kFrames + t) * kBins * 16 + s * 4;
        float4 q[16];
#pragma unroll
        for (int n2 = 0; n2 < 16; ++n2) {
          const int k = 256 * n2 + tid;
          const int bin = k < kBins ? k : (k == kBins ? 0 : kNfft - k);
          q[n2] = *reinterpret_cast<const float4*>(fr + (int64_t)bin * 16);
        }
#pragma unroll
        for (int n2 = 0; n2 < 16; ++n2) {
          const int k = 256 * n2 + tid;
          const float ar = (q[n2].x - o2) * sd, ai = (q[n2].y - o2) * sd;
          const float br = (q[n2].z - o2) * sd, bi = (q[n2].w - o2) * sd;
          cpx z;
          if (n2 < 8) {
            z = k == 0 ? cpx{ar, br}  // irfft ignores the imaginary part of the DC bin
                       : cpx{ar - bi, ai + br};
          } else {
            z = k == kBins ? cpx{0.f, 0.f}        // the zero Nyquist bin
                           : cpx{ar + bi, br - ai};  // Z[N-m] = conj(A[m]) + i conj(B[m])
          }
          v[n2] = z;
        }
      }
      idft16(v);
      {
        // twiddles e^(2 pi i tid k1 / 4096), k1 = 0..15, from four table entries
        cpx wk[16];
        powers16(w_inv(tw, tid), w_inv(tw, 2 * tid), w_inv(tw, 4 * tid), w_inv(tw, 8 * tid), wk);
#pragma unroll
        for (int k1 = 0; k1 < 16; ++k1) {
          const cpx y = k1 == 0 ? v[idft16_slot(0)] : cmul(v[idft16_slot(k1)], wk[k1]);
          bre[k1 * kRow + tid] = y.x;
          bim[k1 * kRow + tid] = y.y;
        }
      }
      __syncthreads();
      {
        // pass 2: thread (k1, c), the 256-point DFT over m = 16 a + c, first level
        const int k1 = tid >> 4, c = tid & 15;
#pragma unroll
        for (int a = 0; a < 16; ++a)
          v[a] = {bre[k1 * kRow + 16 * a + c], bim[k1 * kRow + 16 * a + c]};
        __syncthreads();
        idft16(v);
        // twiddles e^(2 pi i 16 c d / 4096), d = 0..15
        cpx wk[16];
        powers16(w_inv(tw, 16 * c), w_inv(tw, 32 * c), w_inv(tw, 64 * c), w_inv(tw, 128 * c), wk);
#pragma unroll
        for (int d = 0; d < 16; ++d) {
          const cpx u = (d == 0 || c == 0) ? v[idft16_slot(d)] : cmul(v[idft16_slot(d)], wk[d]);
          bre[k1 * kRow + 17 * d + c] = u.x;
          bim[k1 * kRow + 17 * d + c] = u.y;
        }
      }
      __syncthreads();
      {
        // pass 3: thread (d, k1), second level: X[k1 + 16 d + 256 e], e = 0..15
        const int d = tid >> 4, k1 = tid & 15;
#pragma unroll
        for (int c = 0; c < 16; ++c) v[c] = {bre[k1 * kRow + 17 * d + c], bim[k1 * kRow + 17 * d + c]};
        idft16(v);
        const int f = t + 2;
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int hop = f + (e >> 2);
          if (hop >= H0 && hop < H0 + kIstftHops) {
            const int n = k1 + 16 * d + 256 * e;
            const int idx = (hop - H0) * kHop + (n & (kHop - 1));
            const float w = window[n] * inv_n;
            const cpx x = v[idft16_slot(e)];
            acc[idx] += x.x * w;
            acc[AC + idx] += x.y * w;
          }
        }
      }
      __syncthreads();
    }
    // time branch + overlap-add / envelope for this CTA's samples of source s
    const float4 nt = norm_t[b];
    for (int u = tid; u < AC; u += kIstftThreads) {
      const int i = H0 * kHop + u;
      const int j = i - (kPad + kNfft / 2);
      if (j < 0 || j >= kSegment) continue;
      const float env = envelope[i & (kHop - 1)];
      const float2 tv = *reinterpret_cast<const float2*>(time_branch + ((int64_t)b * kSegment + j) * 8 + 2 * s);
      out[((int64_t)b * 8 + 2 * s) * kSegment + j] = (tv.x - nt.w) * nt.z + acc[u] / env;
      out[((int64_t)b * 8 + 2 * s + 1) * kSegment + j] = (tv.y - nt.w) * nt.z + acc[AC + u] / env;
    }
    __syncthreads();
  }
}

}  // namespace

void launch_stft_cac(const float* mix, int B, const float* window, const float2* tw, float* out,
                     double* stats, cudaStream_t s) {
  stft_cac_kernel<<<dim3(kFrames, B), 256, 0, s>>>(mix, window, tw, out, stats);
}

void launch_wave_moments(const float* mix, int B, int64_t n, double* stats, cudaStream_t s) {
  wave_moments_kernel<<<dim3(kWaveMomentBlocks, B), 512, 0, s>>>(mix, n, stats);
}

void launch_norm_finalize(const double* part, int nparts, double count, int B, float4* norm,
                          cudaStream_t s) {
  norm_finalize_kernel<<<(B + 63) / 64, 64, 0, s>>>(part, nparts, count, B, norm);
}

void launch_istft(const float* spec, const float4* norm, const float* window, const float2* tw,
                  const float* envelope, const float* time_branch, const float4* norm_t, float* out,
                  int B, cudaStream_t s) {
  static PerDevice configured;
  if (configured.first())
    cudaFuncSetAttribute(istft_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)kIstftSmem);
  // hops 3 .. 339 of the centred signal hold the segment's samples
  const int groups = (337 + kIstftHops - 1) / kIstftHops;
  istft_kernel<<<dim3(4, groups, B), kIstftThreads, kIstftSmem, s>>>(spec, norm, window, tw,
                                                                     envelope, time_branch, norm_t,
                                                                     out);
}

}  // namespace dmx
