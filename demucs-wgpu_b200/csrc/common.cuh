// Shared device helpers for the HTDemucs v4 sm_100a kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#define DMX_DEVICE __device__ __forceinline__

namespace dmx {

// Once per device for per-context settings such as a kernel's dynamic
// shared-memory limit: a function attribute belongs to the context of the
// device that was current when it was set, so each GPU a process launches on
// needs its own. `first()` is true the first time it is asked on a device.
struct PerDevice {
  std::atomic<uint64_t> done{0};
  bool first() {
    int d = 0;
    cudaGetDevice(&d);
    const uint64_t bit = 1ull << (d & 63);
    return (done.fetch_or(bit) & bit) == 0;
  }
};

constexpr int kSegment = 343980;  // int(39/5 * 44100)
constexpr int kHop = 1024;
constexpr int kNfft = 4096;
constexpr int kBins = 2048;       // Nyquist dropped (spec.rs:101-111)
constexpr int kFrames = 336;      // ceil(343980 / 1024)
constexpr int kPad = 1536;        // hop/2*3 (spec.rs:66)
constexpr int kStftLen = 347136;  // 343980 + 1536 + 1620

// Exact GELU: 0.5 x (1 + erf(x / sqrt 2)) with CUDA's erff.
DMX_DEVICE float gelu(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }
DMX_DEVICE float sigmoid(float g) { return 1.0f / (1.0f + expf(-g)); }

// The tensor-core builds' epilogue activations, in fewer instructions: their
// inputs carry tf32 rounding (2^-11 relative), far above these functions'
// errors. erf by Abramowitz & Stegun, Handbook of Mathematical Functions,
// eq. 7.1.26 (|error| <= 1.5e-7): erf(z) = 1 - t (a1 + t (a2 + t (a3 + t (a4 +
// t a5)))) exp(-z^2), t = 1 / (1 + p z), z >= 0, odd in z; the exponential and
// the reciprocal on the special-function unit.
DMX_DEVICE float erf_as(float z) {
  const float a = fabsf(z);
  const float t = __fdividef(1.0f, fmaf(0.3275911f, a, 1.0f));
  float q = fmaf(1.061405429f, t, -1.453152027f);
  q = fmaf(q, t, 1.421413741f);
  q = fmaf(q, t, -0.284496736f);
  q = fmaf(q, t, 0.254829592f);
  const float r = 1.0f - q * t * __expf(-a * a);
  return copysignf(r, z);
}
DMX_DEVICE float gelu_tc(float x) { return 0.5f * x * (1.0f + erf_as(x * 0.70710678118654752f)); }
// value * sigmoid(gate); 0 once exp(-gate) overflows (gate < -87)
DMX_DEVICE float glu_tc(float value, float gate) { return __fdividef(value, 1.0f + __expf(-gate)); }

// fp32 -> nearest tf32 (ties to even), kept in an fp32 container.
DMX_DEVICE float round_tf32(float x) {
  uint32_t b = __float_as_uint(x);
  b += 0x0FFFu + ((b >> 13) & 1u);
  return __uint_as_float(b & 0xFFFFE000u);
}

// Eight floats from / to a 32-byte-aligned global address in one access
// (sm_100's 256-bit loads and stores): half the requests of two float4s, for
// the per-thread row segments of the tensor-core epilogues.
DMX_DEVICE void ld_global8(const float* p, float* v) {
  asm volatile("ld.global.v8.f32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]),
                 "=f"(v[6]), "=f"(v[7])
               : "l"(p)
               : "memory");
}
DMX_DEVICE void st_global8(float* p, const float* v) {
  asm volatile("st.global.v8.f32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "f"(v[0]),
               "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7])
               : "memory");
}

DMX_DEVICE void st_global8(uint32_t* p, const uint32_t* v) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(v[0]),
               "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}

DMX_DEVICE double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
DMX_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
DMX_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Row statistics held as (sum, sum of squares) in f64, the way the reference
// accumulates GroupNorm / normalisation moments (demucs/ops.rs:564-578).
struct RowNorm {
  float mean, inv;
};
DMX_DEVICE RowNorm row_norm(const double* stats, int row, double count) {
  const double sum = stats[2 * row], sq = stats[2 * row + 1];
  const double mean = sum / count;
  const double var = fmax(sq / count - mean * mean, 0.0);
  RowNorm r;
  r.inv = 1.0f / (float)sqrt(var + 1e-5);
  r.mean = (float)mean;
  return r;
}

}  // namespace dmx
