// CPU ORACLE — TEST INFRASTRUCTURE ONLY.
//
// A C++17/OpenMP restatement of the reference's CPU ("host") HTDemucs v4
// forward and of its chunking / overlap-add / shift driver. It exists to check
// the CUDA path, and as the timed CPU baseline in bench.py. Nothing in the
// product links, loads or calls it: only tests/, __graft_entry__.smoke() and
// bench.py's CPU-baseline leg do, and only as the checker.
//
// Each function names the reference file:line it follows (paths relative to
// the reference project, crates/demucs-core/src/...). The reference is Rust and
// cannot be built in this environment (no cargo, no crates), so the
// restatement is pinned against the reference's own unit-test vectors
// (tests/test_oracle_golden.py) and against PyTorch's primitives
// (tests/test_oracle_torch.py); bitwise equality with the Rust binary is not a
// goal (its FFT/GEMM crates reorder f32 sums).

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>
#include <omp.h>

namespace {

using f32 = float;
using f64 = double;

thread_local std::string g_error;

// ---------------------------------------------------------------------------
// GEMM: C (M x N) = A (M x K) * B (K x N) [+ C], row-major, single-threaded.
// Stands in for the `gemm` 0.18.2 crate (demucs/ops.rs:807-839); the sum order
// differs, which the f32 tolerance absorbs.
// ---------------------------------------------------------------------------
template <int MR, int NR>
inline void micro(int K, const f32* __restrict A, int lda, const f32* __restrict B,
                  int ldb, f32* __restrict C, int ldc, bool acc) {
  f32 c[MR][NR];
  for (int r = 0; r < MR; ++r)
    for (int j = 0; j < NR; ++j) c[r][j] = acc ? C[(size_t)r * ldc + j] : 0.f;
  for (int k = 0; k < K; ++k) {
    const f32* b = B + (size_t)k * ldb;
    for (int r = 0; r < MR; ++r) {
      const f32 a = A[(size_t)r * lda + k];
      for (int j = 0; j < NR; ++j) c[r][j] += a * b[j];
    }
  }
  for (int r = 0; r < MR; ++r)
    for (int j = 0; j < NR; ++j) C[(size_t)r * ldc + j] = c[r][j];
}

inline void micro_edge(int mr, int nr, int K, const f32* A, int lda, const f32* B, int ldb,
                       f32* C, int ldc, bool acc) {
  for (int r = 0; r < mr; ++r)
    for (int j = 0; j < nr; ++j) {
      f32 s = acc ? C[(size_t)r * ldc + j] : 0.f;
      for (int k = 0; k < K; ++k) s += A[(size_t)r * lda + k] * B[(size_t)k * ldb + j];
      C[(size_t)r * ldc + j] = s;
    }
}

void sgemm(int M, int N, int K, const f32* A, int lda, const f32* B, int ldb, f32* C, int ldc,
           bool acc) {
  constexpr int KB = 256;
  for (int k0 = 0; k0 < K; k0 += KB) {
    const int kb = std::min(KB, K - k0);
    const bool a = acc || k0 > 0;
    for (int i = 0; i < M; i += 4) {
      const int mr = std::min(4, M - i);
      for (int j = 0; j < N; j += 32) {
        const int nr = std::min(32, N - j);
        const f32* Ap = A + (size_t)i * lda + k0;
        const f32* Bp = B + (size_t)k0 * ldb + j;
        f32* Cp = C + (size_t)i * ldc + j;
        if (mr == 4 && nr == 32)
          micro<4, 32>(kb, Ap, lda, Bp, ldb, Cp, ldc, a);
        else
          micro_edge(mr, nr, kb, Ap, lda, Bp, ldb, Cp, ldc, a);
      }
    }
  }
}

// Row-parallel GEMM for the big linears.
void sgemm_par(int M, int N, int K, const f32* A, int lda, const f32* B, int ldb, f32* C,
               int ldc) {
  const int block = 32;
#pragma omp parallel for schedule(dynamic)
  for (int i = 0; i < M; i += block) {
    const int m = std::min(block, M - i);
    sgemm(m, N, K, A + (size_t)i * lda, lda, B, ldb, C + (size_t)i * ldc, ldc, false);
  }
}

// ---------------------------------------------------------------------------
// Elementwise maths.
// ---------------------------------------------------------------------------

// erf through the complementary rational approximation the reference uses
// (ops.rs:95-124: the Numerical Recipes `erfcc` Chebyshev fit, fractional
// error < 1.2e-7), evaluated in f32 as there.
f32 erf_ref(f32 x) {
  const f32 z = std::fabs(x);
  const f32 t = 1.0f / (1.0f + 0.5f * z);
  const f32 poly =
      -z * z - 1.26551223f +
      t * (1.00002368f +
           t * (0.37409196f +
                t * (0.09678418f +
                     t * (-0.18628806f +
                          t * (0.27886807f +
                               t * (-1.13520398f +
                                    t * (1.48851587f + t * (-0.82215223f + t * 0.17087277f))))))));
  const f32 tau = t * std::exp(poly);
  const f32 value = 1.0f - tau;
  return x >= 0.f ? value : -value;
}

// Exact GELU (core/ops.rs:95-97).
inline f32 gelu(f32 x) { return 0.5f * x * (1.0f + erf_ref(x * 0.70710678118654752f)); }
inline f32 sigmoid(f32 g) { return 1.0f / (1.0f + std::exp(-g)); }

void gelu_inplace(f32* x, size_t n) {
#pragma omp parallel for schedule(static)
  for (size_t i = 0; i < n; ++i) x[i] = gelu(x[i]);
}

// ---------------------------------------------------------------------------
// Convolutions (demucs/ops.rs:44-211, 299-405, 414-528).
// ---------------------------------------------------------------------------
struct ConvW {
  const f32* w = nullptr;  // PyTorch layout
  const f32* b = nullptr;
  std::vector<int64_t> shape;
  int oc() const { return (int)shape[0]; }
  int ic() const { return (int)shape[1]; }
};

// nn.Conv2d on (B, Cin, H, W) with weight (Cout, Cin, kh, kw); a Conv1d
// weight (Cout, Cin, k) is applied as a (1, k) kernel (ops.rs:52-57).
std::vector<f32> conv2d(const f32* x, int B, int Cin, int H, int W, const ConvW& cw, int sh,
                        int sw, int ph, int pw, int dh, int dw, int* outH, int* outW) {
  int kh, kw;
  if (cw.shape.size() == 3) {
    kh = 1;
    kw = (int)cw.shape[2];
  } else {
    kh = (int)cw.shape[2];
    kw = (int)cw.shape[3];
  }
  const int OC = cw.oc();
  if (cw.ic() != Cin) throw std::runtime_error("conv2d: channel mismatch");
  const int eh = dh * (kh - 1) + 1, ew = dw * (kw - 1) + 1;
  const int Ho = (H + 2 * ph - eh) / sh + 1;
  const int Wo = (W + 2 * pw - ew) / sw + 1;
  const int K = Cin * kh * kw;
  const size_t plane = (size_t)Ho * Wo;
  *outH = Ho;
  *outW = Wo;
  std::vector<f32> out((size_t)B * OC * plane);
  const bool one = kh == 1 && kw == 1 && sh == 1 && sw == 1 && ph == 0 && pw == 0;
  const int NT = 128;
  const size_t tiles = (plane + NT - 1) / NT;
#pragma omp parallel
  {
    std::vector<f32> patch((size_t)K * NT), prod((size_t)OC * NT);
#pragma omp for schedule(dynamic)
    for (long long job = 0; job < (long long)(B * tiles); ++job) {
      const int b = (int)(job / tiles);
      const size_t p0 = (size_t)(job % tiles) * NT;
      const int n = (int)std::min<size_t>(NT, plane - p0);
      const f32* xb = x + (size_t)b * Cin * H * W;
      const f32* src;
      int ldb;
      if (one) {
        src = xb + p0;
        ldb = (int)plane;
      } else {
        for (int k = 0; k < K; ++k) {
          const int ic = k / (kh * kw), tap = k % (kh * kw), ky = tap / kw, kx = tap % kw;
          f32* dst = patch.data() + (size_t)k * NT;
          for (int j = 0; j < n; ++j) {
            const size_t p = p0 + j;
            const int oy = (int)(p / Wo), ox = (int)(p % Wo);
            const int iy = oy * sh + ky * dh - ph, ix = ox * sw + kx * dw - pw;
            dst[j] = (iy < 0 || iy >= H || ix < 0 || ix >= W) ? 0.f
                                                              : xb[((size_t)ic * H + iy) * W + ix];
          }
        }
        src = patch.data();
        ldb = NT;
      }
      sgemm(OC, n, K, cw.w, K, src, ldb, prod.data(), NT, false);
      for (int o = 0; o < OC; ++o) {
        f32* dst = out.data() + ((size_t)b * OC + o) * plane + p0;
        const f32 bias = cw.b[o];
        for (int j = 0; j < n; ++j) dst[j] = prod[(size_t)o * NT + j] + bias;
      }
    }
  }
  return out;
}

// nn.Conv1d on (B, C, T) (ops.rs:367-405).
std::vector<f32> conv1d(const f32* x, int B, int C, int T, const ConvW& cw, int stride, int pad,
                        int dil, int* outT) {
  int h;
  return conv2d(x, B, C, 1, T, cw, 1, stride, 0, pad, 1, dil, &h, outT);
}

// nn.ConvTranspose2d without padding; the caller crops (ops.rs:414-515).
// Weight (Cin, Cout, kh, kw); output starts at the bias and the taps are added
// in tap order, as the reference folds them.
std::vector<f32> conv_transpose2d(const f32* x, int B, int Cin, int H, int W, const ConvW& cw,
                                  int sh, int sw, int* outH, int* outW) {
  int kh, kw;
  if (cw.shape.size() == 3) {
    kh = 1;
    kw = (int)cw.shape[2];
  } else {
    kh = (int)cw.shape[2];
    kw = (int)cw.shape[3];
  }
  if ((int)cw.shape[0] != Cin) throw std::runtime_error("conv_transpose2d: channel mismatch");
  const int OC = (int)cw.shape[1];
  const int Ho = (H - 1) * sh + kh, Wo = (W - 1) * sw + kw;
  *outH = Ho;
  *outW = Wo;
  const int taps = kh * kw;
  // Stacked tap weights: row (tap*OC + co), column ci.
  std::vector<f32> stacked((size_t)taps * OC * Cin);
  for (int ky = 0; ky < kh; ++ky)
    for (int kx = 0; kx < kw; ++kx)
      for (int ci = 0; ci < Cin; ++ci)
        for (int co = 0; co < OC; ++co)
          stacked[((size_t)(ky * kw + kx) * OC + co) * Cin + ci] =
              cw.w[(((size_t)ci * OC + co) * kh + ky) * kw + kx];
  const size_t positions = (size_t)H * W;
  std::vector<f32> out((size_t)B * OC * Ho * Wo);
  for (int b = 0; b < B; ++b) {
    std::vector<f32> product((size_t)taps * OC * positions);
    const f32* xb = x + (size_t)b * Cin * positions;
    const int NT = 256;
    const long long tiles = (long long)((positions + NT - 1) / NT);
#pragma omp parallel
    {
      std::vector<f32> tmp((size_t)taps * OC * NT);
#pragma omp for schedule(dynamic)
      for (long long t = 0; t < tiles; ++t) {
        const size_t p0 = (size_t)t * NT;
        const int n = (int)std::min<size_t>(NT, positions - p0);
        sgemm(taps * OC, n, Cin, stacked.data(), Cin, xb + p0, (int)positions, tmp.data(), NT,
              false);
        for (int r = 0; r < taps * OC; ++r)
          std::memcpy(product.data() + (size_t)r * positions + p0, tmp.data() + (size_t)r * NT,
                      n * sizeof(f32));
      }
    }
#pragma omp parallel for schedule(static)
    for (int co = 0; co < OC; ++co) {
      f32* target = out.data() + ((size_t)b * OC + co) * Ho * Wo;
      for (size_t i = 0; i < (size_t)Ho * Wo; ++i) target[i] = cw.b[co];
      for (int tap = 0; tap < taps; ++tap) {
        const int ky = tap / kw, kx = tap % kw;
        const f32* source = product.data() + ((size_t)tap * OC + co) * positions;
        for (int iy = 0; iy < H; ++iy)
          for (int ix = 0; ix < W; ++ix)
            target[(size_t)(iy * sh + ky) * Wo + ix * sw + kx] += source[(size_t)iy * W + ix];
      }
    }
  }
  return out;
}

// ---------------------------------------------------------------------------
// Norms and gates (demucs/ops.rs:532-743, 930-1094; host.rs:1137-1196).
// ---------------------------------------------------------------------------

// nn.GroupNorm(1, C) over (rows, C, inner): f64 moments, biased variance.
void group_norm1(f32* x, int rows, int C, size_t inner, const f32* w, const f32* b) {
#pragma omp parallel for schedule(dynamic)
  for (int r = 0; r < rows; ++r) {
    f32* s = x + (size_t)r * C * inner;
    const size_t n = (size_t)C * inner;
    f64 sum = 0, sq = 0;
    for (size_t i = 0; i < n; ++i) {
      const f64 v = s[i];
      sum += v;
      sq += v * v;
    }
    const f64 mean = sum / (f64)n;
    const f64 var = std::max(sq / (f64)n - mean * mean, 0.0);
    const f32 inv = 1.0f / (f32)std::sqrt(var + 1e-5);
    const f32 meanf = (f32)mean;
    for (int c = 0; c < C; ++c) {
      const f32 scale = inv * w[c];
      const f32 shift = b[c] - meanf * scale;
      f32* run = s + (size_t)c * inner;
      for (size_t i = 0; i < inner; ++i) run[i] = run[i] * scale + shift;
    }
  }
}

// F.glu(x, dim=1) on (B, 2C, inner) (ops.rs:624-658).
std::vector<f32> glu(const f32* x, int B, int C2, size_t inner) {
  const int C = C2 / 2;
  std::vector<f32> out((size_t)B * C * inner);
#pragma omp parallel for schedule(static)
  for (long long row = 0; row < (long long)B * C; ++row) {
    const int b = (int)(row / C), c = (int)(row % C);
    const f32* v = x + ((size_t)b * C2 + c) * inner;
    const f32* g = v + (size_t)C * inner;
    f32* d = out.data() + (size_t)row * inner;
    for (size_t i = 0; i < inner; ++i) d[i] = v[i] * sigmoid(g[i]);
  }
  return out;
}

// nn.LayerNorm(dim) over rows, f32 statistics (ops.rs:596-621).
std::vector<f32> layer_norm_rows(const f32* x, size_t rows, int dim, const f32* w, const f32* b) {
  std::vector<f32> out(rows * dim);
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < (long long)rows; ++r) {
    const f32* in = x + (size_t)r * dim;
    f32 sum = 0;
    for (int i = 0; i < dim; ++i) sum += in[i];
    const f32 mean = sum / (f32)dim;
    f32 var = 0;
    for (int i = 0; i < dim; ++i) var += (in[i] - mean) * (in[i] - mean);
    var /= (f32)dim;
    const f32 inv = 1.0f / std::sqrt(var + 1e-5f);
    f32* o = out.data() + (size_t)r * dim;
    for (int i = 0; i < dim; ++i) o[i] = (in[i] - mean) * inv * w[i] + b[i];
  }
  return out;
}

// MyGroupNorm(1, C) on a (B, tokens, C) tensor (host.rs:1137-1196).
void group_norm_positions(f32* x, int B, size_t tokens, int C, const f32* w, const f32* b) {
  for (int bi = 0; bi < B; ++bi) {
    f32* s = x + (size_t)bi * tokens * C;
    const size_t n = tokens * C;
    f64 sum = 0, sq = 0;
#pragma omp parallel for reduction(+ : sum, sq) schedule(static)
    for (long long i = 0; i < (long long)n; ++i) {
      const f64 v = s[i];
      sum += v;
      sq += v * v;
    }
    const f64 mean = sum / (f64)n;
    const f64 var = std::max(sq / (f64)n - mean * mean, 0.0);
    const f32 inv = 1.0f / (f32)std::sqrt(var + 1e-5);
    const f32 meanf = (f32)mean;
    std::vector<f32> scale(C), shift(C);
    for (int c = 0; c < C; ++c) {
      scale[c] = inv * w[c];
      shift[c] = b[c] - meanf * scale[c];
    }
#pragma omp parallel for schedule(static)
    for (long long t = 0; t < (long long)tokens; ++t)
      for (int c = 0; c < C; ++c) s[t * C + c] = s[t * C + c] * scale[c] + shift[c];
  }
}

// ---------------------------------------------------------------------------
// Spectrogram front/back end (demucs/spec.rs, dsp/stft.rs).
// ---------------------------------------------------------------------------

// pad1d(x, (left, right), mode='reflect') with the short-input fallback
// (spec.rs:204-236).
std::vector<f32> pad1d_reflect(const f32* x, size_t length, size_t left, size_t right) {
  const size_t max_pad = std::max(left, right);
  size_t extra_left = 0, extra_right = 0;
  if (length <= max_pad) {
    const size_t extra = max_pad - length + 1;
    extra_right = std::min(right, extra);
    extra_left = extra - extra_right;
  }
  const size_t pl = left - extra_left, pr = right - extra_right;
  std::vector<f32> base(extra_left, 0.f);
  base.insert(base.end(), x, x + length);
  base.insert(base.end(), extra_right, 0.f);
  if (base.size() <= pl || base.size() <= pr) throw std::runtime_error("reflect padding too large");
  std::vector<f32> out(base.size() + pl + pr, 0.f);
  std::copy(base.begin(), base.end(), out.begin() + pl);
  for (size_t i = 0; i < pl; ++i) out[pl - 1 - i] = base[i + 1];
  for (size_t i = 0; i < pr; ++i) out[pl + base.size() + i] = base[base.size() - 2 - i];
  return out;
}

// Periodic Hann window (stft.rs:54-61).
std::vector<f32> hann(size_t n) {
  std::vector<f32> w(n);
  for (size_t i = 0; i < n; ++i) w[i] = (f32)(0.5 - 0.5 * std::cos(2.0 * M_PI * (f64)i / (f64)n));
  return w;
}

// In-place radix-2 complex FFT in f64 (sign -1 forward, +1 inverse, no
// scaling). Stands in for rustfft 6.4.1 (stft.rs:90-95, 187, 275).
void fft(std::vector<f64>& re, std::vector<f64>& im, int sign) {
  const size_t n = re.size();
  for (size_t i = 1, j = 0; i < n; ++i) {
    size_t bit = n >> 1;
    for (; j & bit; bit >>= 1) j ^= bit;
    j ^= bit;
    if (i < j) {
      std::swap(re[i], re[j]);
      std::swap(im[i], im[j]);
    }
  }
  for (size_t len = 2; len <= n; len <<= 1) {
    const f64 ang = sign * 2.0 * M_PI / (f64)len;
    for (size_t i = 0; i < n; i += len)
      for (size_t k = 0; k < len / 2; ++k) {
        const f64 wr = std::cos(ang * k), wi = std::sin(ang * k);
        const size_t a = i + k, b = i + k + len / 2;
        const f64 xr = re[b] * wr - im[b] * wi, xi = re[b] * wi + im[b] * wr;
        re[b] = re[a] - xr;
        im[b] = im[a] - xi;
        re[a] += xr;
        im[a] += xi;
      }
  }
}

// torch.stft(center=True, reflect, periodic Hann, optionally normalized) on
// rows of `samples`; out (rows, n/2+1, frames) interleaved complex
// (stft.rs:126-201).
std::vector<f32> stft(const f32* x, int rows, size_t samples, int n_fft, int hop, bool normalized,
                      int* frames_out) {
  const size_t pad = n_fft / 2;
  if (pad >= samples) throw std::runtime_error("reflect padding needs a longer input");
  const size_t padded = samples + 2 * pad;
  const int frames = (int)(1 + (padded - n_fft) / hop);
  const int bins = n_fft / 2 + 1;
  *frames_out = frames;
  const std::vector<f32> window = hann(n_fft);
  const f32 norm = normalized ? 1.0f / std::sqrt((f32)n_fft) : 1.0f;
  std::vector<f32> out((size_t)rows * bins * frames * 2);
#pragma omp parallel
  {
    std::vector<f64> re(n_fft), im(n_fft);
#pragma omp for schedule(dynamic)
    for (long long job = 0; job < (long long)rows * frames; ++job) {
      const int r = (int)(job / frames), f = (int)(job % frames);
      const f32* row = x + (size_t)r * samples;
      for (int i = 0; i < n_fft; ++i) {
        // reflect about both ends without repeating the edge (stft.rs:310-326)
        long long p = (long long)f * hop + i - (long long)pad;
        if (p < 0) p = -p;
        if (p >= (long long)samples) p = 2 * ((long long)samples - 1) - p;
        re[i] = (f64)(row[p] * window[i]);
        im[i] = 0;
      }
      fft(re, im, -1);
      for (int k = 0; k < bins; ++k) {
        f32* o = out.data() + (((size_t)r * bins + k) * frames + f) * 2;
        o[0] = (f32)re[k] * norm;
        o[1] = (f32)im[k] * norm;
      }
    }
  }
  return out;
}

// torch.istft inverse with the window-squared envelope (stft.rs:204-295).
// spec (rows, bins, frames) interleaved complex; returns (rows, length).
std::vector<f32> istft(const f32* spec, int rows, int bins, int frames, int n_fft, int hop,
                       bool normalized, size_t length) {
  const size_t expected = (size_t)n_fft + (size_t)hop * (frames - 1);
  const size_t start = n_fft / 2;
  // length None: hop * (frames - 1) samples (stft.rs:228-232)
  const size_t end = std::min(length == (size_t)-1 ? expected - n_fft / 2 : start + length, expected);
  const size_t out_len = end > start ? end - start : 0;
  const f32 norm_scale = normalized ? std::sqrt((f32)n_fft) : 1.0f;
  const f32 inv_n = norm_scale / (f32)n_fft;
  const std::vector<f32> window = hann(n_fft);
  std::vector<f32> out((size_t)rows * out_len);
#pragma omp parallel
  {
    std::vector<f64> re(n_fft), im(n_fft);
    std::vector<f32> y(expected), env(expected);
#pragma omp for schedule(dynamic)
    for (int r = 0; r < rows; ++r) {
      std::fill(y.begin(), y.end(), 0.f);
      std::fill(env.begin(), env.end(), 0.f);
      for (int f = 0; f < frames; ++f) {
        auto at = [&](int k, int part) {
          return (f64)spec[(((size_t)r * bins + k) * frames + f) * 2 + part];
        };
        re[0] = at(0, 0);
        im[0] = at(0, 1);
        for (int k = 1; k < bins; ++k) {
          re[k] = at(k, 0);
          im[k] = at(k, 1);
          re[n_fft - k] = at(k, 0);
          im[n_fft - k] = -at(k, 1);
        }
        fft(re, im, +1);
        const size_t offset = (size_t)f * hop;
        for (int i = 0; i < n_fft; ++i) {
          const f32 w = window[i];
          y[offset + i] += (f32)re[i] * inv_n * w;
          env[offset + i] += w * w;
        }
      }
      for (size_t i = start; i < end; ++i) {
        const f32 d = env[i];
        out[(size_t)r * out_len + (i - start)] = d != 0.f ? y[i] / d : 0.f;
      }
    }
  }
  return out;
}

// ---------------------------------------------------------------------------
// Model.
// ---------------------------------------------------------------------------
struct Tensor {
  std::vector<f32> v;
  std::vector<int64_t> shape;
};

struct Model {
  std::map<std::string, Tensor> w;
  int segment = 343980;
  const Tensor& get(const std::string& name) const {
    auto it = w.find(name);
    if (it == w.end()) throw std::runtime_error("missing weight " + name);
    return it->second;
  }
  const f32* p(const std::string& name) const { return get(name).v.data(); }
  ConvW conv(const std::string& prefix) const {
    ConvW c;
    const Tensor& t = get(prefix + ".weight");
    c.w = t.v.data();
    c.shape = t.shape;
    c.b = p(prefix + ".bias");
    return c;
  }
};

typedef void (*trace_fn)(const char* name, const f32* data, const int64_t* shape, int ndim,
                         void* user);

struct Tracer {
  trace_fn fn = nullptr;
  void* user = nullptr;
  void operator()(const std::string& name, const std::vector<f32>& v,
                  std::initializer_list<int64_t> shape) const {
    if (!fn) return;
    std::vector<int64_t> s(shape);
    fn(name.c_str(), v.data(), s.data(), (int)s.size(), user);
  }
};

// (b, c, f, t) -> (b*f, c, t) and back (ops.rs:1517-1581).
std::vector<f32> to_leading_freq(const f32* x, int B, int C, int F, int T) {
  std::vector<f32> out((size_t)B * F * C * T);
#pragma omp parallel for schedule(static)
  for (long long row = 0; row < (long long)B * F; ++row) {
    const int b = (int)(row / F), f = (int)(row % F);
    for (int c = 0; c < C; ++c)
      std::memcpy(out.data() + ((size_t)row * C + c) * T, x + (((size_t)b * C + c) * F + f) * T,
                  T * sizeof(f32));
  }
  return out;
}
std::vector<f32> from_leading_freq(const f32* x, int B, int C, int F, int T) {
  std::vector<f32> out((size_t)B * C * F * T);
#pragma omp parallel for schedule(static)
  for (long long bc = 0; bc < (long long)B * C; ++bc) {
    const int b = (int)(bc / C), c = (int)(bc % C);
    for (int f = 0; f < F; ++f)
      std::memcpy(out.data() + ((size_t)bc * F + f) * T, x + (((size_t)b * F + f) * C + c) * T,
                  T * sizeof(f32));
  }
  return out;
}

// DConv residual branch on (rows, C, T) (host.rs:985-1059, with the fused tail
// of ops.rs:930-1094 — same arithmetic as the unfused operators).
void dconv(const Model& m, const std::string& prefix, std::vector<f32>& x, int rows, int C, int T) {
  for (int d = 0; d < 2; ++d) {
    const std::string at = prefix + ".dconv.layers." + std::to_string(d);
    const int dil = 1 << d;
    const ConvW c1 = m.conv(at + ".0");
    const int hidden = c1.oc();
    int To;
    std::vector<f32> y = conv1d(x.data(), rows, C, T, c1, 1, dil, dil, &To);
    group_norm1(y.data(), rows, hidden, T, m.p(at + ".1.weight"), m.p(at + ".1.bias"));
    gelu_inplace(y.data(), y.size());
    const ConvW c2 = m.conv(at + ".3");
    std::vector<f32> z = conv1d(y.data(), rows, hidden, T, c2, 1, 0, 1, &To);
    const f32* nw = m.p(at + ".4.weight");
    const f32* nb = m.p(at + ".4.bias");
    const f32* gamma = m.p(at + ".6.scale");
#pragma omp parallel for schedule(dynamic)
    for (int r = 0; r < rows; ++r) {
      const f32* s = z.data() + (size_t)r * 2 * C * T;
      const size_t n = (size_t)2 * C * T;
      f64 sum = 0, sq = 0;
      for (size_t i = 0; i < n; ++i) {
        const f64 v = s[i];
        sum += v;
        sq += v * v;
      }
      const f64 mean = sum / (f64)n;
      const f64 var = std::max(sq / (f64)n - mean * mean, 0.0);
      const f32 inv = 1.0f / (f32)std::sqrt(var + 1e-5);
      const f32 meanf = (f32)mean;
      f32* dst = x.data() + (size_t)r * C * T;
      for (int k = 0; k < C; ++k) {
        const f32 vs = inv * nw[k], vsh = nb[k] - meanf * vs;
        const f32 gs = inv * nw[k + C], gsh = nb[k + C] - meanf * gs;
        const f32* values = s + (size_t)k * T;
        const f32* gates = s + (size_t)(k + C) * T;
        for (int i = 0; i < T; ++i) {
          const f32 value = values[i] * vs + vsh;
          const f32 gate = gates[i] * gs + gsh;
          dst[(size_t)k * T + i] += gamma[k] * (value * sigmoid(gate));
        }
      }
    }
  }
}

// Linear: x (rows, in) -> (rows, out), weight (out, in) (core/ops.rs:14-58).
std::vector<f32> linear(const f32* x, size_t rows, int in, const f32* w, const f32* b, int out) {
  std::vector<f32> wt((size_t)in * out);
  for (int o = 0; o < out; ++o)
    for (int i = 0; i < in; ++i) wt[(size_t)i * out + o] = w[(size_t)o * in + i];
  std::vector<f32> y(rows * out);
  sgemm_par((int)rows, out, in, x, in, wt.data(), out, y.data(), out);
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < (long long)rows; ++r)
    for (int o = 0; o < out; ++o) y[r * out + o] += b[o];
  return y;
}

// softmax(q k^T * scale) v for one head with the deferred normalisation
// (ops.rs:1350-1408, 1442-1458). q (nq, d), k/v (nk, d), out (nq, d).
void attention_head(const f32* q, const f32* k, const f32* v, int nq, int nk, int d, f32 scale,
                    f32* out) {
  std::vector<f32> qs((size_t)nq * d), kt((size_t)d * nk), s((size_t)nq * nk);
  for (size_t i = 0; i < (size_t)nq * d; ++i) qs[i] = q[i] * scale;
  for (int j = 0; j < nk; ++j)
    for (int c = 0; c < d; ++c) kt[(size_t)c * nk + j] = k[(size_t)j * d + c];
  sgemm(nq, nk, d, qs.data(), d, kt.data(), nk, s.data(), nk, false);
  std::vector<f32> sums(nq);
  for (int i = 0; i < nq; ++i) {
    f32* row = s.data() + (size_t)i * nk;
    f32 mx = -INFINITY;
    for (int j = 0; j < nk; ++j) mx = std::max(mx, row[j]);
    f32 sum = 0;
    for (int j = 0; j < nk; ++j) {
      row[j] = std::exp(row[j] - mx);
      sum += row[j];
    }
    sums[i] = sum;
  }
  sgemm(nq, d, nk, s.data(), nk, v, d, out, d, false);
  for (int i = 0; i < nq; ++i)
    if (sums[i] > 0.f) {
      const f32 inv = 1.0f / sums[i];
      for (int c = 0; c < d; ++c) out[(size_t)i * d + c] *= inv;
    }
}

// nn.MultiheadAttention, batch_first (host.rs:1199-1312).
std::vector<f32> mha(const Model& m, const std::string& attn, const f32* query, const f32* key,
                     int B, int nq, int nk, int dim, int heads) {
  const f32* w = m.p(attn + ".in_proj_weight");
  const f32* bias = m.p(attn + ".in_proj_bias");
  const size_t dd = (size_t)dim * dim;
  std::vector<f32> q = linear(query, (size_t)B * nq, dim, w, bias, dim);
  std::vector<f32> k = linear(key, (size_t)B * nk, dim, w + dd, bias + dim, dim);
  std::vector<f32> v = linear(key, (size_t)B * nk, dim, w + 2 * dd, bias + 2 * dim, dim);
  const int dh = dim / heads;
  const f32 scale = 1.0f / std::sqrt((f32)dh);
  std::vector<f32> merged((size_t)B * nq * dim);
#pragma omp parallel for schedule(dynamic)
  for (int bh = 0; bh < B * heads; ++bh) {
    const int b = bh / heads, h = bh % heads;
    std::vector<f32> qh((size_t)nq * dh), kh((size_t)nk * dh), vh((size_t)nk * dh),
        oh((size_t)nq * dh);
    for (int i = 0; i < nq; ++i)
      std::memcpy(&qh[(size_t)i * dh], &q[((size_t)b * nq + i) * dim + h * dh], dh * 4);
    for (int i = 0; i < nk; ++i) {
      std::memcpy(&kh[(size_t)i * dh], &k[((size_t)b * nk + i) * dim + h * dh], dh * 4);
      std::memcpy(&vh[(size_t)i * dh], &v[((size_t)b * nk + i) * dim + h * dh], dh * 4);
    }
    attention_head(qh.data(), kh.data(), vh.data(), nq, nk, dh, scale, oh.data());
    for (int i = 0; i < nq; ++i)
      std::memcpy(&merged[((size_t)b * nq + i) * dim + h * dh], &oh[(size_t)i * dh], dh * 4);
  }
  return linear(merged.data(), (size_t)B * nq, dim, m.p(attn + ".out_proj.weight"),
                m.p(attn + ".out_proj.bias"), dim);
}

// One transformer layer, self (host.rs:1315-1365) or cross (1368-1429).
std::vector<f32> transformer_layer(const Model& m, const std::string& at, bool cross,
                                   const std::vector<f32>& x, const std::vector<f32>* other,
                                   int B, int n, int n_other, int dim, int hidden,
                                   const Tracer& trace) {
  const size_t rows = (size_t)B * n;
  std::vector<f32> nq = layer_norm_rows(x.data(), rows, dim, m.p(at + ".norm1.weight"),
                                        m.p(at + ".norm1.bias"));
  std::vector<f32> att;
  if (cross) {
    std::vector<f32> nk = layer_norm_rows(other->data(), (size_t)B * n_other, dim,
                                          m.p(at + ".norm2.weight"), m.p(at + ".norm2.bias"));
    att = mha(m, at + ".cross_attn", nq.data(), nk.data(), B, n, n_other, dim, 8);
  } else {
    att = mha(m, at + ".self_attn", nq.data(), nq.data(), B, n, n, dim, 8);
  }
  const f32* g1 = m.p(at + ".gamma_1.scale");
  const f32* g2 = m.p(at + ".gamma_2.scale");
  std::vector<f32> out(rows * dim);
  for (size_t r = 0; r < rows; ++r)
    for (int c = 0; c < dim; ++c) out[r * dim + c] = x[r * dim + c] + att[r * dim + c] * g1[c];
  const std::string norm = cross ? ".norm3" : ".norm2";
  std::vector<f32> normed =
      layer_norm_rows(out.data(), rows, dim, m.p(at + norm + ".weight"), m.p(at + norm + ".bias"));
  std::vector<f32> h =
      linear(normed.data(), rows, dim, m.p(at + ".linear1.weight"), m.p(at + ".linear1.bias"), hidden);
  gelu_inplace(h.data(), h.size());
  std::vector<f32> fed =
      linear(h.data(), rows, hidden, m.p(at + ".linear2.weight"), m.p(at + ".linear2.bias"), dim);
  for (size_t r = 0; r < rows; ++r)
    for (int c = 0; c < dim; ++c) out[r * dim + c] = out[r * dim + c] + fed[r * dim + c] * g2[c];
  group_norm_positions(out.data(), B, n, dim, m.p(at + ".norm_out.weight"),
                       m.p(at + ".norm_out.bias"));
  trace(at, out, {B, n, dim});
  return out;
}

// create_2d_sin_embedding flattened to (frame*freq + bin, dim) (host.rs:1078-1106).
std::vector<f32> pos2d(int dim, int height, int width, f32 max_period) {
  const int half = dim / 2, pairs = half / 2;
  const f32 log_period = std::log(max_period) / (f32)half;
  std::vector<f32> div(pairs);
  for (int j = 0; j < pairs; ++j) div[j] = std::exp(-((f32)(2 * j)) * log_period);
  std::vector<f32> out((size_t)width * height * dim);
  for (int t = 0; t < width; ++t)
    for (int f = 0; f < height; ++f) {
      f32* o = out.data() + ((size_t)t * height + f) * dim;
      for (int j = 0; j < pairs; ++j) {
        const f32 w = (f32)t * div[j], h = (f32)f * div[j];
        o[2 * j] = std::sin(w);
        o[2 * j + 1] = std::cos(w);
        o[half + 2 * j] = std::sin(h);
        o[half + 2 * j + 1] = std::cos(h);
      }
    }
  return out;
}

// create_sin_embedding (host.rs:1110-1122).
std::vector<f32> pos1d(int length, int dim, f32 max_period) {
  const int half = dim / 2;
  std::vector<f32> out((size_t)length * dim);
  for (int t = 0; t < length; ++t)
    for (int i = 0; i < half; ++i) {
      const f32 exponent = (f32)i / ((f32)half - 1.0f);
      const f32 phase = (f32)t / std::pow(max_period, exponent);
      out[(size_t)t * dim + i] = std::cos(phase);
      out[(size_t)t * dim + half + i] = std::sin(phase);
    }
  return out;
}

f32 mean_f64(const f32* v, size_t n) {
  f64 s = 0;
  for (size_t i = 0; i < n; ++i) s += v[i];
  return (f32)(s / (f64)n);
}

// torch.std(unbiased=True), two-pass in f64 (ops.rs:1494-1509).
f32 std_unbiased(const f32* v, size_t n) {
  if (n < 2) return NAN;
  f64 s = 0;
  for (size_t i = 0; i < n; ++i) s += v[i];
  const f64 mean = s / (f64)n;
  f64 acc = 0;
  for (size_t i = 0; i < n; ++i) {
    const f64 d = (f64)v[i] - mean;
    acc += d * d;
  }
  return (f32)std::sqrt(acc / (f64)(n - 1));
}

// Htdemucs::forward (host.rs:202-520). mix (B, 2, length <= segment) ->
// out (B, 4, 2, length).
void forward(const Model& m, const f32* mix, int B, int length, f32* result,
             const Tracer& trace) {
  const int L = m.segment;
  if (length > L) throw std::runtime_error("input longer than the training segment");
  const int C_AUDIO = 2, S = 4, hop = 1024, nfft = 4096;
  std::vector<f32> padded((size_t)B * C_AUDIO * L, 0.f);
  for (int b = 0; b < B; ++b)
    for (int c = 0; c < C_AUDIO; ++c)
      std::memcpy(&padded[((size_t)b * C_AUDIO + c) * L], mix + ((size_t)b * C_AUDIO + c) * length,
                  length * sizeof(f32));

  // _spec (spec.rs:62-113)
  const int le = (L + hop - 1) / hop;
  const int pad = hop / 2 * 3;
  const int right = pad + le * hop - L;
  const size_t plen = (size_t)L + pad + right;
  std::vector<f32> rows((size_t)B * C_AUDIO * plen);
  for (int r = 0; r < B * C_AUDIO; ++r) {
    std::vector<f32> p = pad1d_reflect(&padded[(size_t)r * L], L, pad, right);
    std::memcpy(&rows[(size_t)r * plen], p.data(), plen * sizeof(f32));
  }
  int frames;
  std::vector<f32> spec = stft(rows.data(), B * C_AUDIO, plen, nfft, hop, true, &frames);
  if (frames != le + 4) throw std::runtime_error("unexpected frame count");
  const int bins = nfft / 2 + 1, F0 = nfft / 2;
  // CaC pack (spec.rs:240-254): channel 2c = re, 2c+1 = im; frames [2, 2+le).
  std::vector<f32> x((size_t)B * 4 * F0 * le);
  for (int b = 0; b < B; ++b)
    for (int c = 0; c < C_AUDIO; ++c)
      for (int f = 0; f < F0; ++f)
        for (int t = 0; t < le; ++t) {
          const f32* z = &spec[((((size_t)b * C_AUDIO + c) * bins + f) * frames + t + 2) * 2];
          x[(((size_t)b * 4 + 2 * c) * F0 + f) * le + t] = z[0];
          x[(((size_t)b * 4 + 2 * c + 1) * F0 + f) * le + t] = z[1];
        }
  trace("_magnitude", x, {B, 4, F0, le});

  // Per-batch normalisation (host.rs:250-261, 523-543).
  std::vector<f32> mean(B), sd(B), mean_t(B), sd_t(B);
  std::vector<f32> xt = padded;
  const size_t xn = (size_t)4 * F0 * le, tn = (size_t)C_AUDIO * L;
  for (int b = 0; b < B; ++b) {
    mean[b] = mean_f64(&x[b * xn], xn);
    sd[b] = std_unbiased(&x[b * xn], xn);
    mean_t[b] = mean_f64(&padded[b * tn], tn);
    sd_t[b] = std_unbiased(&padded[b * tn], tn);
    const f32 s1 = 1.0f / (1e-5f + sd[b]);
    for (size_t i = 0; i < xn; ++i) x[b * xn + i] = (x[b * xn + i] - mean[b]) * s1;
    const f32 s2 = 1.0f / (1e-5f + sd_t[b]);
    for (size_t i = 0; i < tn; ++i) xt[b * tn + i] = (xt[b * tn + i] - mean_t[b]) * s2;
  }
  trace("x_normalized", x, {B, 4, F0, le});
  trace("xt_normalized", xt, {B, C_AUDIO, L});

  std::vector<std::vector<f32>> saved, saved_t;
  std::vector<int> saved_c, saved_f, lengths_t, saved_tc, saved_tl;
  int C = 4, F = F0, T = le, Ct = C_AUDIO, Tt = L;
  for (int i = 0; i < 4; ++i) {
    const std::string ti = "tencoder." + std::to_string(i);
    // time_encoder_forward (host.rs:625-678)
    lengths_t.push_back(Tt);
    {
      std::vector<f32> in = xt;
      int Tin = Tt;
      if (Tt % 4 != 0) {
        Tin = Tt + (4 - Tt % 4);
        in.assign((size_t)B * Ct * Tin, 0.f);
        for (size_t r = 0; r < (size_t)B * Ct; ++r)
          std::memcpy(&in[r * Tin], &xt[r * Tt], Tt * sizeof(f32));
      }
      const ConvW cw = m.conv(ti + ".conv");
      int To;
      std::vector<f32> y = conv1d(in.data(), B, Ct, Tin, cw, 4, 2, 1, &To);
      gelu_inplace(y.data(), y.size());
      const int Co = cw.oc();
      dconv(m, ti, y, B, Co, To);
      const ConvW rw = m.conv(ti + ".rewrite");
      int T2;
      std::vector<f32> r = conv1d(y.data(), B, Co, To, rw, 1, 0, 1, &T2);
      xt = glu(r.data(), B, 2 * Co, To);
      Ct = Co;
      Tt = To;
    }
    trace(ti, xt, {B, Ct, Tt});
    saved_t.push_back(xt);
    saved_tc.push_back(Ct);
    saved_tl.push_back(Tt);

    // freq_encoder_forward (host.rs:577-622)
    const std::string fi = "encoder." + std::to_string(i);
    {
      const ConvW cw = m.conv(fi + ".conv");
      int Fo, To;
      std::vector<f32> y = conv2d(x.data(), B, C, F, T, cw, 4, 1, 2, 0, 1, 1, &Fo, &To);
      gelu_inplace(y.data(), y.size());
      const int Co = cw.oc();
      std::vector<f32> flat = to_leading_freq(y.data(), B, Co, Fo, To);
      dconv(m, fi, flat, B * Fo, Co, To);
      y = from_leading_freq(flat.data(), B, Co, Fo, To);
      const ConvW rw = m.conv(fi + ".rewrite");
      int F2, T2;
      std::vector<f32> r = conv2d(y.data(), B, Co, Fo, To, rw, 1, 1, 0, 0, 1, 1, &F2, &T2);
      x = glu(r.data(), B, 2 * Co, (size_t)Fo * To);
      C = Co;
      F = Fo;
      T = To;
    }
    trace(fi, x, {B, C, F, T});
    if (i == 0) {
      // add_frequency_embedding (host.rs:546-574): 0.2 * (10 * emb)[f, c]
      const Tensor& emb = m.get("freq_emb.embedding.weight");
      const f32 scale = 0.2f;
      for (int b = 0; b < B; ++b)
        for (int c = 0; c < C; ++c)
          for (int f = 0; f < F; ++f) {
            const f32 value = scale * (emb.v[(size_t)f * C + c] * 10.0f);
            f32* run = &x[(((size_t)b * C + c) * F + f) * T];
            for (int t = 0; t < T; ++t) run[t] += value;
          }
      trace("encoder.0.post_emb", x, {B, C, F, T});
    }
    saved.push_back(x);
    saved_c.push_back(C);
    saved_f.push_back(F);
  }

  // channel_upsampler (host.rs:320-338): linear over channels per (f, t).
  const int D = 512, Fb = F, Tb = T;
  const int ntok = Fb * Tb;
  auto channel_mix = [&](const std::vector<f32>& in, int b_, int cin, int positions,
                         const std::string& name, int cout) {
    // (b, cin, positions) -> (b, cout, positions)
    std::vector<f32> out((size_t)b_ * cout * positions);
    const Tensor& wt = m.get(name + ".weight");
    const f32* bias = m.p(name + ".bias");
    for (int b = 0; b < b_; ++b) {
      std::vector<f32> flat((size_t)positions * cin);
      for (int c = 0; c < cin; ++c)
        for (int p = 0; p < positions; ++p)
          flat[(size_t)p * cin + c] = in[((size_t)b * cin + c) * positions + p];
      std::vector<f32> y = linear(flat.data(), positions, cin, wt.v.data(), bias, cout);
      for (int c = 0; c < cout; ++c)
        for (int p = 0; p < positions; ++p)
          out[((size_t)b * cout + c) * positions + p] = y[(size_t)p * cout + c];
    }
    return out;
  };
  std::vector<f32> xu = channel_mix(x, B, C, ntok, "channel_upsampler", D);
  std::vector<f32> xtu = channel_mix(xt, B, Ct, Tt, "channel_upsampler_t", D);
  trace("channel_upsampler", xu, {B, D, ntok});
  trace("channel_upsampler_t", xtu, {B, D, Tt});

  // transformer_forward (host.rs:830-946)
  std::vector<f32> spec_tok((size_t)B * ntok * D), time_tok((size_t)B * Tt * D);
  for (int b = 0; b < B; ++b) {
    for (int c = 0; c < D; ++c)
      for (int f = 0; f < Fb; ++f)
        for (int t = 0; t < Tb; ++t)
          spec_tok[((size_t)b * ntok + (size_t)t * Fb + f) * D + c] =
              xu[(((size_t)b * D + c) * Fb + f) * Tb + t];
    for (int c = 0; c < D; ++c)
      for (int t = 0; t < Tt; ++t)
        time_tok[((size_t)b * Tt + t) * D + c] = xtu[((size_t)b * D + c) * Tt + t];
  }
  const std::vector<f32> p2 = pos2d(D, Fb, Tb, 10000.0f);
  const std::vector<f32> p1 = pos1d(Tt, D, 10000.0f);
  spec_tok = layer_norm_rows(spec_tok.data(), (size_t)B * ntok, D,
                             m.p("crosstransformer.norm_in.weight"),
                             m.p("crosstransformer.norm_in.bias"));
  for (int b = 0; b < B; ++b)
    for (size_t i = 0; i < (size_t)ntok * D; ++i) spec_tok[b * (size_t)ntok * D + i] += p2[i] * 1.0f;
  time_tok = layer_norm_rows(time_tok.data(), (size_t)B * Tt, D,
                             m.p("crosstransformer.norm_in_t.weight"),
                             m.p("crosstransformer.norm_in_t.bias"));
  for (int b = 0; b < B; ++b)
    for (size_t i = 0; i < (size_t)Tt * D; ++i) time_tok[b * (size_t)Tt * D + i] += p1[i] * 1.0f;
  trace("crosstransformer.in#0", spec_tok, {B, ntok, D});
  trace("crosstransformer.in#1", time_tok, {B, Tt, D});
  for (int l = 0; l < 5; ++l) {
    const bool cross = l % 2 == 1;
    const std::string a = "crosstransformer.layers." + std::to_string(l);
    const std::string at = "crosstransformer.layers_t." + std::to_string(l);
    if (cross) {
      std::vector<f32> old = spec_tok;
      spec_tok = transformer_layer(m, a, true, spec_tok, &time_tok, B, ntok, Tt, D, 2048, trace);
      time_tok = transformer_layer(m, at, true, time_tok, &old, B, Tt, ntok, D, 2048, trace);
    } else {
      spec_tok = transformer_layer(m, a, false, spec_tok, nullptr, B, ntok, ntok, D, 2048, trace);
      time_tok = transformer_layer(m, at, false, time_tok, nullptr, B, Tt, Tt, D, 2048, trace);
    }
  }
  // back to (b, c, f, t) and (b, c, t)
  for (int b = 0; b < B; ++b) {
    for (int c = 0; c < D; ++c)
      for (int f = 0; f < Fb; ++f)
        for (int t = 0; t < Tb; ++t)
          xu[(((size_t)b * D + c) * Fb + f) * Tb + t] =
              spec_tok[((size_t)b * ntok + (size_t)t * Fb + f) * D + c];
    for (int c = 0; c < D; ++c)
      for (int t = 0; t < Tt; ++t)
        xtu[((size_t)b * D + c) * Tt + t] = time_tok[((size_t)b * Tt + t) * D + c];
  }
  x = channel_mix(xu, B, D, ntok, "channel_downsampler", C);
  xt = channel_mix(xtu, B, D, Tt, "channel_downsampler_t", Ct);
  trace("channel_downsampler", x, {B, C, ntok});
  trace("channel_downsampler_t", xt, {B, Ct, Tt});

  // Decoders, execution order e = 0..3 (checkpoint index 3 - e).
  for (int e = 0; e < 4; ++e) {
    const bool last = e == 3;
    const int j = 3 - e;
    // freq_decoder_forward (host.rs:682-759)
    {
      const std::string dn = "decoder." + std::to_string(j);
      const std::vector<f32> skip = saved.back();
      saved.pop_back();
      for (size_t i = 0; i < x.size(); ++i) x[i] = x[i] + skip[i];
      const ConvW rw = m.conv(dn + ".rewrite");
      int F2, T2;
      std::vector<f32> r = conv2d(x.data(), B, C, F, T, rw, 1, 1, 1, 1, 1, 1, &F2, &T2);
      std::vector<f32> g = glu(r.data(), B, 2 * C, (size_t)F * T);
      std::vector<f32> flat = to_leading_freq(g.data(), B, C, F, T);
      dconv(m, dn, flat, B * F, C, T);
      std::vector<f32> pre = from_leading_freq(flat.data(), B, C, F, T);
      const ConvW tw = m.conv(dn + ".conv_tr");
      int Fu, Tu;
      std::vector<f32> up = conv_transpose2d(pre.data(), B, C, F, T, tw, 4, 1, &Fu, &Tu);
      const int Co = (int)tw.shape[1];
      const int cut = 2;
      const int Fo = Fu - 2 * cut;
      x.assign((size_t)B * Co * Fo * T, 0.f);
      for (int b = 0; b < B; ++b)
        for (int c = 0; c < Co; ++c)
          for (int f = 0; f < Fo; ++f)
            std::memcpy(&x[(((size_t)b * Co + c) * Fo + f) * T],
                        &up[(((size_t)b * Co + c) * Fu + f + cut) * Tu], T * sizeof(f32));
      if (!last) gelu_inplace(x.data(), x.size());
      C = Co;
      F = Fo;
      trace(dn, x, {B, C, F, T});
    }
    // time_decoder_forward (host.rs:763-827)
    {
      const std::string dn = "tdecoder." + std::to_string(j);
      const std::vector<f32> skip = saved_t.back();
      saved_t.pop_back();
      const int length_t = lengths_t.back();
      lengths_t.pop_back();
      for (size_t i = 0; i < xt.size(); ++i) xt[i] = xt[i] + skip[i];
      const ConvW rw = m.conv(dn + ".rewrite");
      int T2;
      std::vector<f32> r = conv1d(xt.data(), B, Ct, Tt, rw, 1, 1, 1, &T2);
      std::vector<f32> g = glu(r.data(), B, 2 * Ct, Tt);
      dconv(m, dn, g, B, Ct, Tt);
      const ConvW tw = m.conv(dn + ".conv_tr");
      int Hu, Tu;
      std::vector<f32> up = conv_transpose2d(g.data(), B, Ct, 1, Tt, tw, 1, 4, &Hu, &Tu);
      const int Co = (int)tw.shape[1];
      const int cut = 2;
      if (cut + length_t > Tu) throw std::runtime_error("transposed conv too short");
      xt.assign((size_t)B * Co * length_t, 0.f);
      for (size_t r2 = 0; r2 < (size_t)B * Co; ++r2)
        std::memcpy(&xt[r2 * length_t], &up[r2 * Tu + cut], length_t * sizeof(f32));
      if (!last) gelu_inplace(xt.data(), xt.size());
      Ct = Co;
      Tt = length_t;
      trace(dn, xt, {B, Ct, Tt});
    }
  }

  // Denormalise the freq branch, unpack, pad, _ispec (host.rs:466-497).
  const size_t fn = (size_t)16 * F * T;
  for (int b = 0; b < B; ++b) {
    const f32 offset = mean[b], scale = sd[b];
    const f32 o2 = -offset / scale;
    for (size_t i = 0; i < fn; ++i) x[b * fn + i] = (x[b * fn + i] - o2) * scale;
  }
  const int bins2 = F + 1, frames2 = T + 4;
  std::vector<f32> z((size_t)B * S * C_AUDIO * bins2 * frames2 * 2, 0.f);
  for (int b = 0; b < B; ++b)
    for (int s = 0; s < S; ++s)
      for (int c = 0; c < C_AUDIO; ++c) {
        const size_t row = ((size_t)b * S + s) * C_AUDIO + c;
        const f32* re = &x[(((size_t)b * 16) + s * 4 + c * 2) * F * T];
        const f32* im = re + (size_t)F * T;
        for (int f = 0; f < F; ++f)
          for (int t = 0; t < T; ++t) {
            f32* o = &z[((row * bins2 + f) * frames2 + t + 2) * 2];
            o[0] = re[(size_t)f * T + t];
            o[1] = im[(size_t)f * T + t];
          }
      }
  const size_t ilen = (size_t)hop * le + 2 * pad;
  std::vector<f32> wav =
      istft(z.data(), B * S * C_AUDIO, bins2, frames2, nfft, hop, true, ilen);
  // time branch: (B, 8, L) -> (B, 4, 2, L), denormalised; sum (host.rs:499-519)
  for (int b = 0; b < B; ++b) {
    const f32 offset = mean_t[b], scale = sd_t[b];
    const f32 o2 = -offset / scale;
    for (int r = 0; r < S * C_AUDIO; ++r) {
      const f32* w = &wav[((size_t)b * S * C_AUDIO + r) * ilen + pad];
      const f32* tb = &xt[((size_t)b * S * C_AUDIO + r) * L];
      f32* o = result + ((size_t)b * S * C_AUDIO + r) * length;
      for (int i = 0; i < length; ++i) o[i] = (tb[i] - o2) * scale + w[i];
    }
  }
}

// ---------------------------------------------------------------------------
// Separation driver (streaming.rs:52-400, pipeline.rs:105-151, 380-515,
// mix.rs:552-633). The forward is a callback so tests can plug in an
// identity forward (tests/streaming_ola.rs:62-90) or the CUDA path.
// ---------------------------------------------------------------------------
typedef int (*segment_fn)(const f32* padded, int group, int segment, f32* out, void* user);

struct ShiftRng {
  uint64_t s;
  explicit ShiftRng(uint64_t seed) : s(seed * 6364136223846793005ULL + 1ULL) {}
  uint64_t randint(uint64_t max) {
    s = s * 6364136223846793005ULL + 1442695040888963407ULL;
    return (s >> 33) % (max + 1);
  }
};

std::vector<f32> transition_weight(int segment, f64 power) {
  const int half = segment / 2;
  std::vector<f32> w;
  w.reserve(segment);
  for (int i = 1; i <= half; ++i) w.push_back((f32)i);
  for (int i = segment - half; i >= 1; --i) w.push_back((f32)i);
  f32 mx = 0.f;
  for (f32 v : w) mx = std::max(mx, v);
  mx = std::max(mx, 1.0f);
  for (f32& v : w) v = std::pow(v / mx, (f32)power);
  return w;
}

// TensorChunk.padded over the (optionally shifted) view of the mix: centre a
// `chunk`-sample window starting at view index `vstart` inside `segment`
// samples, zero outside the view and outside the mix (mix.rs:552-633).
void padded_chunk(const f32* mix, int channels, int64_t length, int64_t shift_offset,
                  int64_t max_shift, int64_t vstart, int64_t chunk, int segment, f32* out) {
  const int64_t view_length = max_shift ? length + max_shift - shift_offset : length;
  const int64_t start = vstart - (segment - chunk) / 2;
  for (int c = 0; c < channels; ++c)
    for (int i = 0; i < segment; ++i) {
      const int64_t v = start + i;
      f32 sample = 0.f;
      if (v >= 0 && v < view_length) {
        const int64_t mi = max_shift ? shift_offset + v - max_shift : v;
        if (mi >= 0 && mi < length) sample = mix[(size_t)c * length + mi];
      }
      out[(size_t)c * segment + i] = sample;
    }
}

// center_trim(tensor, reference) (pipeline.rs:105-113): the first kept
// sample of a `length`-sample signal trimmed to `reference`; the larger half
// of an odd excess is removed at the end.
int64_t center_trim_start(int64_t length, int64_t reference) {
  return length <= reference ? 0 : (length - reference) / 2;
}

// One streaming split pass over the (optionally shifted) normalised mix;
// returns (sources, 2, view_length) OLA-finalised output in view coordinates.
int split_pass(const f32* mix, int64_t length, int segment, f64 overlap, f64 power, int batch,
               int64_t shift_offset, int64_t max_shift, segment_fn fwd, void* user,
               std::vector<f32>& view_out, int64_t* view_len_out) {
  const int S = 4, CH = 2;
  const int64_t stride = (int64_t)((1.0 - overlap) * (f64)segment);
  if (stride == 0) throw std::runtime_error("overlap leaves a zero stride");
  const std::vector<f32> weight = transition_weight(segment, power);
  const int64_t view_length = max_shift ? length + max_shift - shift_offset : length;
  *view_len_out = view_length;
  view_out.assign((size_t)S * CH * view_length, 0.f);
  std::vector<f32> sum_w(view_length, 0.f);
  std::vector<int64_t> starts;
  for (int64_t o = 0; o < view_length; o += stride) starts.push_back(o);
  std::vector<f32> batched, outb;
  for (size_t g0 = 0; g0 < starts.size(); g0 += batch) {
    const int group = (int)std::min<size_t>(batch, starts.size() - g0);
    batched.assign((size_t)group * CH * segment, 0.f);
    for (int slot = 0; slot < group; ++slot) {
      const int64_t vstart = starts[g0 + slot];
      const int64_t chunk = std::min<int64_t>(view_length - vstart, segment);
      padded_chunk(mix, CH, length, shift_offset, max_shift, vstart, chunk, segment,
                   &batched[(size_t)slot * CH * segment]);
    }
    outb.assign((size_t)group * S * CH * segment, 0.f);
    if (fwd(batched.data(), group, segment, outb.data(), user) != 0) return 1;
    for (int slot = 0; slot < group; ++slot) {
      const int64_t vstart = starts[g0 + slot];
      const int64_t chunk = std::min<int64_t>(view_length - vstart, segment);
      const int64_t trim = center_trim_start(segment, chunk);
      for (int r = 0; r < S * CH; ++r) {
        const f32* src = &outb[((size_t)slot * S * CH + r) * segment + trim];
        f32* dst = &view_out[(size_t)r * view_length + vstart];
        for (int64_t t = 0; t < chunk; ++t) dst[t] += weight[t] * src[t];
      }
      for (int64_t t = 0; t < chunk; ++t) sum_w[vstart + t] += weight[t];
    }
  }
  for (int64_t t = 0; t < view_length; ++t) {
    if (sum_w[t] <= 0.f) throw std::runtime_error("overlap-add left a sample with no weight");
    for (int r = 0; r < S * CH; ++r) view_out[(size_t)r * view_length + t] /= sum_w[t];
  }
  return 0;
}

}  // namespace

// ---------------------------------------------------------------------------
// C API (ctypes).
// ---------------------------------------------------------------------------
extern "C" {

const char* orc_last_error() { return g_error.c_str(); }

int orc_threads(int n) {
  if (n > 0) omp_set_num_threads(n);
  return omp_get_max_threads();
}

void* orc_create(int segment) {
  Model* m = new Model();
  m->segment = segment;
  return m;
}
void orc_destroy(void* h) { delete static_cast<Model*>(h); }

int orc_set(void* h, const char* name, const float* data, const int64_t* shape, int ndim) {
  Model* m = static_cast<Model*>(h);
  Tensor t;
  size_t n = 1;
  for (int i = 0; i < ndim; ++i) {
    t.shape.push_back(shape[i]);
    n *= (size_t)shape[i];
  }
  t.v.assign(data, data + n);
  m->w[name] = std::move(t);
  return 0;
}

int orc_forward(void* h, const float* mix, int B, int length, float* out, trace_fn fn,
                void* user) {
  try {
    Tracer tr{fn, user};
    forward(*static_cast<Model*>(h), mix, B, length, out, tr);
    return 0;
  } catch (const std::exception& e) {
    g_error = e.what();
    return 1;
  }
}

// Global normalisation of a (2, length) mix (streaming.rs:52-85):
// ref = channel mean; mean, unbiased std + 1e-8 in f64.
void orc_scan_norm(const float* mix, int channels, int64_t length, float* mean_out,
                   float* std_out) {
  const f64 count = (f64)length;
  f64 sum = 0, sq = 0;
  for (int64_t t = 0; t < length; ++t) {
    f64 acc = 0;
    for (int c = 0; c < channels; ++c) acc += (f64)mix[(size_t)c * length + t];
    const f64 r = acc / channels;
    sum += r;
    sq += r * r;
  }
  const f64 mean = sum / count;
  const f64 var = count > 1 ? (sq - sum * sum / count) / (count - 1) : 0.0;
  *mean_out = (f32)mean;
  *std_out = (f32)std::sqrt(std::max(var, 0.0)) + 1e-8f;
}

// Whole-track separation: normalise, shift passes, split passes, OLA,
// denormalise (api.rs:520-785, pipeline.rs:380-515). mix (2, length) raw;
// stems (4, 2, length).
int orc_separate(const float* mix_raw, int64_t length, int segment, int shifts, double overlap,
                 double power, int batch, segment_fn fwd, void* user, float* stems) {
  try {
    const int S = 4, CH = 2;
    f32 mean, sd;
    orc_scan_norm(mix_raw, CH, length, &mean, &sd);
    std::vector<f32> mix((size_t)CH * length);
    for (size_t i = 0; i < mix.size(); ++i) mix[i] = (mix_raw[i] - mean) / sd;
    std::vector<f32> acc((size_t)S * CH * length, 0.f);
    std::vector<f32> view;
    int64_t vlen;
    if (shifts == 0) {
      if (split_pass(mix.data(), length, segment, overlap, power, batch, 0, 0, fwd, user, view,
                     &vlen))
        return 1;
      acc = view;
    } else {
      const int64_t max_shift = (int64_t)(0.5 * 44100.0);
      ShiftRng rng(0x5eed1234ULL);
      const f32 scale = 1.0f / (f32)shifts;
      for (int pass = 0; pass < shifts; ++pass) {
        const int64_t offset = (int64_t)rng.randint((uint64_t)max_shift);
        const int64_t trim = max_shift - offset;
        if (split_pass(mix.data(), length, segment, overlap, power, batch, offset, max_shift, fwd,
                       user, view, &vlen))
          return 1;
        for (int r = 0; r < S * CH; ++r)
          for (int64_t t = 0; t < length; ++t) {
            const int64_t tv = t + trim;
            if (tv < vlen) {
              if (shifts == 1)
                acc[(size_t)r * length + t] = view[(size_t)r * vlen + tv] * scale;
              else
                acc[(size_t)r * length + t] += view[(size_t)r * vlen + tv];
            }
          }
      }
      if (shifts > 1)
        for (f32& v : acc) v = v * scale;
    }
    for (size_t i = 0; i < acc.size(); ++i) stems[i] = acc[i] * sd + mean;
    return 0;
  } catch (const std::exception& e) {
    g_error = e.what();
    return 1;
  }
}

// --- single ops, for the known-answer tests ---
int orc_conv1d(const float* x, int B, int C, int T, const float* w, const float* b, int oc, int k,
               int stride, int pad, int dil, float* out, int* out_t) {
  ConvW cw;
  cw.w = w;
  cw.b = b;
  cw.shape = {oc, C, k};
  std::vector<f32> y = conv1d(x, B, C, T, cw, stride, pad, dil, out_t);
  std::memcpy(out, y.data(), y.size() * sizeof(f32));
  return 0;
}
int orc_conv2d(const float* x, int B, int C, int H, int W, const float* w, const float* b, int oc,
               int kh, int kw, int sh, int sw, int ph, int pw, float* out, int* oh, int* ow) {
  ConvW cw;
  cw.w = w;
  cw.b = b;
  cw.shape = {oc, C, kh, kw};
  std::vector<f32> y = conv2d(x, B, C, H, W, cw, sh, sw, ph, pw, 1, 1, oh, ow);
  std::memcpy(out, y.data(), y.size() * sizeof(f32));
  return 0;
}
int orc_conv_transpose1d(const float* x, int B, int C, int T, const float* w, const float* b,
                         int oc, int k, int stride, float* out, int* out_t) {
  ConvW cw;
  cw.w = w;
  cw.b = b;
  cw.shape = {C, oc, k};
  int h;
  std::vector<f32> y = conv_transpose2d(x, B, C, 1, T, cw, 1, stride, &h, out_t);
  std::memcpy(out, y.data(), y.size() * sizeof(f32));
  return 0;
}
int orc_group_norm1(float* x, int rows, int C, int inner, const float* w, const float* b) {
  group_norm1(x, rows, C, inner, w, b);
  return 0;
}
int orc_layer_norm(const float* x, int rows, int dim, const float* w, const float* b, float* out) {
  std::vector<f32> y = layer_norm_rows(x, rows, dim, w, b);
  std::memcpy(out, y.data(), y.size() * sizeof(f32));
  return 0;
}
int orc_glu(const float* x, int B, int C2, int inner, float* out) {
  std::vector<f32> y = glu(x, B, C2, inner);
  std::memcpy(out, y.data(), y.size() * sizeof(f32));
  return 0;
}
float orc_gelu(float x) { return gelu(x); }
int orc_attention_head(const float* q, const float* k, const float* v, int nq, int nk, int d,
                       float scale, float* out) {
  attention_head(q, k, v, nq, nk, d, scale, out);
  return 0;
}
float orc_std_unbiased(const float* v, int n) { return std_unbiased(v, n); }
int orc_hann(int n, float* out) {
  std::vector<f32> w = hann(n);
  std::memcpy(out, w.data(), n * sizeof(f32));
  return 0;
}
int orc_reflect_pad(const float* x, int n, int left, int right, float* out) {
  std::vector<f32> y = pad1d_reflect(x, n, left, right);
  std::memcpy(out, y.data(), y.size() * sizeof(f32));
  return (int)y.size();
}
int orc_stft(const float* x, int rows, int samples, int n_fft, int hop, int normalized,
             float* out, int* frames) {
  try {
    std::vector<f32> y = stft(x, rows, samples, n_fft, hop, normalized != 0, frames);
    std::memcpy(out, y.data(), y.size() * sizeof(f32));
    return 0;
  } catch (const std::exception& e) {
    g_error = e.what();
    return 1;
  }
}
int orc_istft(const float* spec, int rows, int bins, int frames, int n_fft, int hop,
              int normalized, int length, float* out) {
  std::vector<f32> y = istft(spec, rows, bins, frames, n_fft, hop, normalized != 0,
                             length < 0 ? (size_t)-1 : (size_t)length);
  std::memcpy(out, y.data(), y.size() * sizeof(f32));
  return (int)(y.size() / rows);
}
// center_trim of rows x length to rows x reference (pipeline.rs:105-113).
int orc_center_trim(const float* x, int rows, int64_t length, int64_t reference, float* out) {
  const int64_t keep = std::min(length, reference), start = center_trim_start(length, reference);
  for (int r = 0; r < rows; ++r)
    for (int64_t t = 0; t < keep; ++t) out[(size_t)r * keep + t] = x[(size_t)r * length + start + t];
  return (int)keep;
}

int orc_transition_weight(int segment, double power, float* out) {
  std::vector<f32> w = transition_weight(segment, power);
  std::memcpy(out, w.data(), w.size() * sizeof(f32));
  return 0;
}
uint64_t orc_shift_randint(uint64_t seed, int draws, uint64_t max, uint64_t* out) {
  ShiftRng r(seed);
  for (int i = 0; i < draws; ++i) out[i] = r.randint(max);
  return 0;
}
int orc_pos2d(int dim, int height, int width, float max_period, float* out) {
  std::vector<f32> y = pos2d(dim, height, width, max_period);
  std::memcpy(out, y.data(), y.size() * sizeof(f32));
  return 0;
}
int orc_padded_chunk(const float* mix, int channels, int64_t length, int64_t shift_offset,
                     int64_t max_shift, int64_t vstart, int64_t chunk, int segment, float* out) {
  padded_chunk(mix, channels, length, shift_offset, max_shift, vstart, chunk, segment, out);
  return 0;
}
int orc_pos1d(int length, int dim, float max_period, float* out) {
  std::vector<f32> y = pos1d(length, dim, max_period);
  std::memcpy(out, y.data(), y.size() * sizeof(f32));
  return 0;
}
}
