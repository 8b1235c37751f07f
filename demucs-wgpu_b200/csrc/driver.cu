// Separation driver on the device (streaming.rs:52-400, pipeline.rs:105-151,
// 380-515, mix.rs:552-633): global normalisation of the track, centred chunk
// extraction from the (shifted) view, triangular overlap-add and the final
// divide / trim / denormalise. The sums are formed in the reference's order
// (chunks in increasing index), so the result does not depend on how the
// chunks were grouped into forwards or spread over GPUs.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace dmx {

namespace {

constexpr int kNormBlocks = 296;  // fixed grid: the f64 partials are summed in block order
constexpr int kNormThreads = 512;

// One sample of the channel-mean signal added to a thread's running moments
// (streaming.rs:52-67: r = (l + r) / 2 in f64). Every moment pass uses this
// one definition, so a pass over windows reproduces a whole-track pass.
DMX_DEVICE void moments_add(double& s, double& q, float left, float right) {
  const double r = ((double)left + (double)right) / 2.0;
  s += r;
  q = __fma_rn(r, r, q);
}

// The block's threads' moments summed (warps, then the warp sums in order)
// into partials[2 * block].
DMX_DEVICE void block_moments(double s, double q, double* __restrict__ partials) {
  __shared__ double red[2][32];
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
      partials[2 * blockIdx.x] = s;
      partials[2 * blockIdx.x + 1] = q;
    }
  }
}

// mean, std (+1e-8) of the channel-mean signal from the block partials, summed
// in block order (streaming.rs:68-77)
DMX_DEVICE float2 norm_from_partials(const double* __restrict__ partials, int nparts, int64_t n) {
  double sum = 0.0, sq = 0.0;
  for (int i = 0; i < nparts; ++i) {
    sum += partials[2 * i];
    sq += partials[2 * i + 1];
  }
  const double count = (double)n;
  const double mean = sum / count;
  const double var = count > 1.0 ? (sq - sum * sum / count) / (count - 1.0) : 0.0;
  return make_float2((float)mean, (float)sqrt(fmax(var, 0.0)) + 1e-8f);
}

// Per-block moments of the channel-mean signal, written to partials[2*block]
// (no atomics, so the result does not depend on scheduling).
__global__ void track_partials_kernel(const float* __restrict__ left,
                                      const float* __restrict__ right, int64_t n,
                                      double* __restrict__ partials) {
  double s = 0.0, q = 0.0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    moments_add(s, q, left[i], right[i]);
  block_moments(s, q, partials);
}

// (x - mean) / std into mix_norm (2, n) (streaming.rs:81-85), after the
// moments (streaming.rs:52-78).
__global__ void track_normalize_kernel(const float* __restrict__ left,
                                       const float* __restrict__ right, int64_t n,
                                       const double* __restrict__ partials, int nparts,
                                       float* __restrict__ mix_norm, float2* __restrict__ norm) {
  __shared__ float2 s_norm;
  if (threadIdx.x == 0) {
    s_norm = norm_from_partials(partials, nparts, n);
    if (blockIdx.x == 0) *norm = s_norm;
  }
  __syncthreads();
  const float meanf = s_norm.x, sd = s_norm.y;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    mix_norm[i] = (left[i] - meanf) / sd;
    mix_norm[n + i] = (right[i] - meanf) / sd;
  }
}

// The moments pass over a track read in windows: thread k of the
// kNormBlocks x kNormThreads grid keeps its running moments in state[2k..]
// and adds the window's samples k, k + grid, ... in order. Every window
// starts at a multiple of the grid size, so each thread sees exactly the
// samples, in the order, that track_partials_kernel's thread k sees.
__global__ void moments_window_kernel(const float* __restrict__ left,
                                      const float* __restrict__ right, int64_t count,
                                      double* __restrict__ state) {
  const int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  double s = state[2 * k], q = state[2 * k + 1];
  for (int64_t i = k; i < count; i += (int64_t)gridDim.x * blockDim.x) moments_add(s, q, left[i], right[i]);
  state[2 * k] = s;
  state[2 * k + 1] = q;
}

__global__ void moments_final_kernel(const double* __restrict__ state, double* __restrict__ partials) {
  const int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  block_moments(state[2 * k], state[2 * k + 1], partials);
}

__global__ void norm_kernel(const double* __restrict__ partials, int nparts, int64_t n,
                            float2* __restrict__ norm) {
  *norm = norm_from_partials(partials, nparts, n);
}

// (x - mean) / std in place over rows of a window (the normalisation of
// track_normalize_kernel, sample for sample)
__global__ void normalize_window_kernel(float* __restrict__ x, int64_t ld, int64_t count,
                                        const float2* __restrict__ norm) {
  const float2 nz = *norm;
  float* row = x + (int64_t)blockIdx.y * ld;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count;
       i += (int64_t)gridDim.x * blockDim.x)
    row[i] = (row[i] - nz.x) / nz.y;
}

// segment: the samples each chunk is cut to (its window and the OLA weights);
// row: the samples of one forward row (the model's training length). A chunk
// shorter than a row (a `segment` override) is centred in `segment` samples
// and zero padded at the end of the row, as Htdemucs::forward pads a short
// input (host.rs:217-229); only the row's first `segment` output samples are
// used.
// The buffers' windows: the normalised mix holds samples [mix_lo, mix_lo +
// mix_n) in rows of mix_ld; the accumulator view samples from acc_lo in rows
// of acc_ld; stems, output sample t at column t - out_lo in rows of out_ld.
struct ChunkGeom {
  int64_t length, view_length, shift_offset, max_shift, stride;
  int segment, row;
  int64_t mix_lo, mix_ld, mix_n, acc_lo, acc_ld, out_lo, out_ld;
};

DMX_DEVICE int64_t chunk_len(const ChunkGeom& g, int64_t c) {
  const int64_t start = c * g.stride;
  const int64_t rest = g.view_length - start;
  return rest < g.segment ? rest : g.segment;
}

__global__ void gather_chunks_kernel(const float* __restrict__ mix_norm, ChunkGeom g,
                                     int64_t chunk0, float* __restrict__ out) {
  const int slot = blockIdx.y, c = blockIdx.z;
  const int64_t chunk = chunk0 + slot;
  const int64_t vstart = chunk * g.stride;
  const int64_t len = chunk_len(g, chunk);
  const int64_t start = vstart - (g.segment - len) / 2;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < g.row;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t v = start + i;
    float sample = 0.f;
    if (i < g.segment && v >= 0 && v < g.view_length) {
      const int64_t mi = g.max_shift ? g.shift_offset + v - g.max_shift : v;
      const int64_t wi = mi - g.mix_lo;
      if (mi >= 0 && mi < g.length && wi >= 0 && wi < g.mix_n) sample = mix_norm[(int64_t)c * g.mix_ld + wi];
    }
    out[((int64_t)slot * 2 + c) * g.row + i] = sample;
  }
}

// acc (8, view_hi - view_lo) += weight * trimmed chunk output, chunks
// [chunk0, chunk0 + count) in increasing order per sample.
__global__ void ola_accumulate_kernel(const float* __restrict__ chunks, ChunkGeom g,
                                      int64_t chunk0, int count, const float* __restrict__ weight,
                                      float* __restrict__ acc, int64_t view_lo, int64_t view_hi) {
  const int64_t first = chunk0 * g.stride;
  const int64_t last_c = chunk0 + count - 1;
  const int64_t end = last_c * g.stride + chunk_len(g, last_c);
  const int64_t v = first + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (v >= end || v < view_lo || v >= view_hi) return;
  int64_t chi = v / g.stride;
  if (chi > last_c) chi = last_c;
  int64_t clo = chi - (g.segment + g.stride - 1) / g.stride;
  if (clo < chunk0) clo = chunk0;
  float vals[8];
#pragma unroll
  for (int r = 0; r < 8; ++r) vals[r] = acc[(int64_t)r * (view_hi - view_lo) + (v - view_lo)];
  for (int64_t c = clo; c <= chi; ++c) {
    const int64_t u = v - c * g.stride;
    const int64_t len = chunk_len(g, c);
    if (u < 0 || u >= len) continue;
    const int64_t trim = (g.segment - len) / 2;
    const float w = weight[u];
    const float* src = chunks + (c - chunk0) * 8 * (int64_t)g.row + trim + u;
    // product and sum rounded separately, as the reference's `acc += w * x` does
    // (no contraction into an FMA): each contribution is round(w * x), so a sample's
    // two contributions sum to the same bits in either order, and a sharded run's
    // boundary merge (acc + tail) reproduces the one-GPU sum exactly
#pragma unroll
    for (int r = 0; r < 8; ++r) vals[r] = __fadd_rn(vals[r], __fmul_rn(w, src[(int64_t)r * g.row]));
  }
#pragma unroll
  for (int r = 0; r < 8; ++r) acc[(int64_t)r * (view_hi - view_lo) + (v - view_lo)] = vals[r];
}

// mode 0: stems = (acc/sw) * std + mean            (shifts == 0)
// mode 1: stems = ((acc/sw) * scale) * std + mean  (shifts == 1)
// mode 2: pass  += acc/sw                          (one of several shifts)
// mode 3: stems = (pass * scale) * std + mean      (after the last shift)
// mode 4: stems = acc/sw                           (one of several shifts, summed by the caller)
// Every product and sum is rounded on its own, as the reference's f32 loops
// (streaming.rs:219-260, pipeline.rs:60-67) round them: no FMA contraction.
__global__ void ola_finish_kernel(const float* __restrict__ acc, ChunkGeom g, int64_t trim,
                                  const float* __restrict__ weight, const float2* __restrict__ norm,
                                  float scale, int mode, float* __restrict__ pass,
                                  float* __restrict__ stems, int64_t t_lo, int64_t t_hi) {
  const int64_t t = t_lo + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= t_hi || t >= g.length) return;
  const float2 nz = *norm;
  float* out = stems + (t - g.out_lo);
  if (mode == 3) {
#pragma unroll
    for (int r = 0; r < 8; ++r)
      out[(int64_t)r * g.out_ld] =
          __fadd_rn(__fmul_rn(__fmul_rn(pass[(int64_t)r * g.length + t], scale), nz.y), nz.x);
    return;
  }
  const int64_t v = t + trim;
  if (v >= g.view_length) return;
  const int64_t nchunks = (g.view_length + g.stride - 1) / g.stride;
  int64_t chi = v / g.stride;
  if (chi > nchunks - 1) chi = nchunks - 1;
  int64_t clo = chi - (g.segment + g.stride - 1) / g.stride;
  if (clo < 0) clo = 0;
  float sw = 0.f;
  for (int64_t c = clo; c <= chi; ++c) {
    const int64_t u = v - c * g.stride;
    if (u >= 0 && u < chunk_len(g, c)) sw += weight[u];
  }
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const float y = acc[(int64_t)r * g.acc_ld + (v - g.acc_lo)] / sw;
    if (mode == 0) out[(int64_t)r * g.out_ld] = __fadd_rn(__fmul_rn(y, nz.y), nz.x);
    else if (mode == 1)
      out[(int64_t)r * g.out_ld] = __fadd_rn(__fmul_rn(__fmul_rn(y, scale), nz.y), nz.x);
    else if (mode == 4) out[(int64_t)r * g.out_ld] = y;
    else pass[(int64_t)r * g.length + t] = __fadd_rn(pass[(int64_t)r * g.length + t], y);
  }
}

}  // namespace

void launch_track_normalize(const float* left, const float* right, int64_t n, double* scratch,
                            float* mix_norm, float2* norm, cudaStream_t s) {
  track_partials_kernel<<<kNormBlocks, kNormThreads, 0, s>>>(left, right, n, scratch);
  track_normalize_kernel<<<kNormBlocks, kNormThreads, 0, s>>>(left, right, n, scratch, kNormBlocks,
                                                              mix_norm, norm);
}

int track_normalize_scratch_doubles() { return 2 * kNormBlocks; }

void launch_track_normalize_blocks(const float* left, const float* right, int64_t n, int blocks,
                                   double* scratch, float* mix_norm, float2* norm, cudaStream_t s) {
  track_partials_kernel<<<blocks, kNormThreads, 0, s>>>(left, right, n, scratch);
  track_normalize_kernel<<<blocks, kNormThreads, 0, s>>>(left, right, n, scratch, blocks, mix_norm, norm);
}

int64_t moments_grid() { return (int64_t)kNormBlocks * kNormThreads; }
int64_t moments_state_doubles() { return 2 * moments_grid() + 2 * kNormBlocks; }

void launch_moments_window(const float* left, const float* right, int64_t count, double* state,
                           cudaStream_t s) {
  moments_window_kernel<<<kNormBlocks, kNormThreads, 0, s>>>(left, right, count, state);
}

void launch_moments_final(double* state, int64_t n, float2* norm, cudaStream_t s) {
  double* partials = state + 2 * moments_grid();
  moments_final_kernel<<<kNormBlocks, kNormThreads, 0, s>>>(state, partials);
  norm_kernel<<<1, 1, 0, s>>>(partials, kNormBlocks, n, norm);
}

void launch_normalize_window(float* x, int64_t ld, int64_t count, const float2* norm, cudaStream_t s) {
  if (count <= 0) return;
  const unsigned blocks = (unsigned)std::min<int64_t>((count + 1023) / 1024, 148 * 2);
  normalize_window_kernel<<<dim3(blocks, 2), 1024, 0, s>>>(x, ld, count, norm);
}

static ChunkGeom geom(int64_t length, int64_t shift_offset, int64_t max_shift, int segment,
                      int64_t stride, int row = 0, const DriverWindow* win = nullptr) {
  ChunkGeom g;
  g.row = row > 0 ? row : segment;
  g.length = length;
  g.shift_offset = shift_offset;
  g.max_shift = max_shift;
  g.view_length = max_shift ? length + max_shift - shift_offset : length;
  g.stride = stride;
  g.segment = segment;
  g.mix_lo = win ? win->mix_lo : 0;
  g.mix_ld = win ? win->mix_ld : length;
  g.mix_n = win ? win->mix_n : length;
  g.acc_lo = win ? win->acc_lo : 0;
  g.acc_ld = win ? win->acc_ld : g.view_length;
  g.out_lo = win ? win->out_lo : 0;
  g.out_ld = win ? win->out_ld : length;
  return g;
}

void launch_gather_chunks(const float* mix_norm, int64_t length, int64_t shift_offset,
                          int64_t max_shift, int segment, int64_t stride, int64_t chunk0,
                          int count, float* out, cudaStream_t s, int row, const DriverWindow* win) {
  const ChunkGeom g = geom(length, shift_offset, max_shift, segment, stride, row, win);
  gather_chunks_kernel<<<dim3(84, count, 2), 1024, 0, s>>>(mix_norm, g, chunk0, out);
}

void launch_ola_accumulate(const float* chunks, int64_t length, int64_t shift_offset,
                           int64_t max_shift, int segment, int64_t stride, int64_t chunk0,
                           int count, const float* weight, float* acc, int64_t view_lo,
                           int64_t view_hi, cudaStream_t s, int row) {
  const ChunkGeom g = geom(length, shift_offset, max_shift, segment, stride, row);
  const int64_t span = (count - 1) * stride + segment;
  ola_accumulate_kernel<<<(unsigned)((span + 255) / 256), 256, 0, s>>>(
      chunks, g, chunk0, count, weight, acc, view_lo, view_hi);
}

void launch_ola_finish(const float* acc, int64_t length, int64_t shift_offset, int64_t max_shift,
                       int segment, int64_t stride, const float* weight, const float2* norm,
                       float scale, int mode, float* pass, float* stems, cudaStream_t s,
                       int64_t t_lo, int64_t t_hi, const DriverWindow* win) {
  const ChunkGeom g = geom(length, shift_offset, max_shift, segment, stride, 0, win);
  const int64_t trim = max_shift ? max_shift - shift_offset : 0;
  if (t_hi < 0 || t_hi > length) t_hi = length;
  if (t_lo < 0) t_lo = 0;
  if (t_hi <= t_lo) return;
  ola_finish_kernel<<<(unsigned)((t_hi - t_lo + 255) / 256), 256, 0, s>>>(
      acc, g, trim, weight, norm, scale, mode, pass, stems, t_lo, t_hi);
}

}  // namespace dmx
