// Launchers of the sm_100a kernels (host side). All take the stream to
// enqueue on; none synchronises.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace dmx {

// Sets the thread-local message dmx_last_error() returns (abi.cu).
void set_last_error(const char* msg);

// spectral.cu. The moments come as partials (sum, sum of squares; f64):
// launch_stft_cac writes B * kFrames of them (one per segment and frame),
// launch_wave_moments B * kWaveMomentBlocks; launch_norm_finalize adds a
// segment's `nparts` partials in order.
constexpr int kWaveMomentBlocks = 148;
void launch_stft_cac(const float* mix, int B, const float* window, const float2* tw, float* out,
                     double* stats, cudaStream_t s);
void launch_wave_moments(const float* mix, int B, int64_t n, double* stats, cudaStream_t s);
void launch_norm_finalize(const double* part, int nparts, double count, int B, float4* norm,
                          cudaStream_t s);
void launch_istft(const float* spec, const float4* norm, const float* window, const float2* tw,
                  const float* envelope, const float* time_branch, const float4* norm_t, float* out,
                  int B, cudaStream_t s);

// dconv.cu — one DConv layer on x (rows, T, C) channels-last, in place.
// Weights as packed for the GEMM path: w1[(k*C + c)*w1_ld + h] (k = tap),
// w2[h*w2_ld + 2c] value / [h*w2_ld + 2c + 1] gate, b2 likewise interleaved;
// n2w/n2b in the reference's order (value c, gate c + C). Rows longer than
// one tile need y (rows*T*C/8 floats) and part1/part2 (rows*tiles*2 doubles).
struct DConvArgs {
  float* x;
  int C, rows, T, dil, tiles;
  const float* w1;
  int w1_ld;
  const float* b1;
  const float* n1w;
  const float* n1b;
  const float* w2;
  int w2_ld;
  const float* b2;
  const float* n2w;
  const float* n2b;
  const float* gamma;
  float* y;
  double* part1;
  double* part2;
  int* err;  // raised when a bounded wait gives up
  int round_out;  // store the updated x rounded to nearest tf32 (it feeds only tf32 GEMMs)
  // tensor-core path: single-pass tf32 (x read by the tensor core as tf32, the
  // weights' high parts only) instead of 3xTF32; the BF16 build's choice
  int single;
  // tensor-core path (dconv_tc.cu): K-major weights rounded to nearest tf32
  // ([w1_npad][3C], [w2_npad][16]) and their residuals w - tf32(w)
  const float* w1_tc;
  const float* w1_tc_lo;
  int w1_npad;
  const float* w2_tc;
  const float* w2_tc_lo;
  int w2_npad;
  // host memory, dconv_tc_const_floats(C) floats: v and the packed upper
  // triangle of M (off-diagonal doubled; dconv_tc_slot order) for the moments
  // of conv2's output, then conv1's bias and GroupNorm1's weight and bias
  const float* zq_host;
  // device memory, dconv_zq_floats(C) floats: the same moments for the SIMT
  // kernels over g~ = (g_0 .. g_{C/8-1}, 1) with conv2's bias as the last
  // input: v, then M row by row, each of dconv_zq_stride(C) floats (zero padded)
  const float* zq_dev;
};
inline int dconv_zq_stride(int C) { return (C / 8 + 1 + 3) / 4 * 4; }
inline int dconv_zq_floats(int C) { return dconv_zq_stride(C) * (C / 8 + 2); }
// K slot (of 16) of conv2 input i in the tensor-core weight copies of the
// narrow layers: hidden channels i < hid/2 at slot i, the others at
// 8 + i - hid/2, and i == hid (the constant-1 bias input) at slot 15.
inline int dconv_tc_slot(int hid, int i) {
  return i < hid / 2 ? i : (i < hid ? 8 + i - hid / 2 : 15);
}
int dconv_tiles(int T);
bool dconv_row_fused(int T);
bool launch_dconv(const DConvArgs& a, cudaStream_t s);
// Row moments of z = conv2(GELU(GroupNorm1(y))) into st2 (rows x 2 doubles)
// from y (rows*T, ld) and its moments st1, by the quadratic form over zq
// (DConvArgs::zq_dev); C 192 or 384 (dconv.cu). `part` holds
// rows * dconv_zstats_parts(T) partials (2 doubles each), added in order.
int dconv_zstats_parts(int T);
bool launch_dconv_zstats(int C, const float* y, int ld, int rows, int T, const float* n1w,
                         const float* n1b, const double* st1, double* st2, double* part,
                         const float* zq, cudaStream_t s);
// tensor-core DConv widths: C 48 and 96 (3xTF32 or single-pass), C 192
// (single-pass only)
bool dconv_tc_supported(int C, int T, bool single);
// work items per row of the tensor-core DConv (rows of more than one need
// part1/part2 and y: rows*T*dconv_tc_ystride(C) floats)
int dconv_tc_tiles(int T);
int dconv_tc_ystride(int C);
int dconv_tc_const_floats(int C);
bool launch_dconv_tc(const DConvArgs& a, cudaStream_t s);

// transformer.cu
// round_out: store the output rounded to nearest tf32 (when it feeds only tf32 GEMMs);
// out16: store it as bf16 there instead of `out` (when it feeds only bf16 GEMMs)
void launch_layer_norm(const float* x, int64_t rows, int ntok, const float* w, const float* b,
                       const float* pos, float* out, cudaStream_t s, bool round_out = false,
                       uint16_t* out16 = nullptr);
void launch_group_norm_apply(float* x, int B, int64_t ntok, const double* stats, const float* w,
                             const float* b, cudaStream_t s);
void launch_flash_attention(const float* q, int ldq, const float* k, const float* v, int ldkv,
                            float* o, int ldo, int B, int heads, int nq, int nk, float scale,
                            cudaStream_t s);

// driver.cu
// scratch: track_normalize_scratch_doubles() doubles of per-block partials
void launch_track_normalize(const float* left, const float* right, int64_t n, double* scratch,
                            float* mix_norm, float2* norm, cudaStream_t s);
int track_normalize_scratch_doubles();
// The same two kernels on `blocks` blocks; scratch holds 2*blocks doubles.
void launch_track_normalize_blocks(const float* left, const float* right, int64_t n, int blocks,
                                   double* scratch, float* mix_norm, float2* norm, cudaStream_t s);
// The moments of a track read in windows: state holds moments_state_doubles()
// doubles, zeroed before the first window; every window but the last holds a
// multiple of moments_grid() samples. launch_moments_final writes the same
// (mean, std) launch_track_normalize computes for the whole track.
int64_t moments_grid();
int64_t moments_state_doubles();
void launch_moments_window(const float* left, const float* right, int64_t count, double* state,
                           cudaStream_t s);
void launch_moments_final(double* state, int64_t n, float2* norm, cudaStream_t s);
// (x - mean) / std in place over two rows of `count` samples, `ld` apart
void launch_normalize_window(float* x, int64_t ld, int64_t count, const float2* norm, cudaStream_t s);
// Windowed buffers of the streaming driver (NULL: whole-track buffers): the
// normalised mix holds samples [mix_lo, mix_lo + mix_n) in rows of mix_ld;
// the accumulator holds view samples from acc_lo in rows of acc_ld; finished
// sample t goes to column t - out_lo of rows out_ld apart.
struct DriverWindow {
  int64_t mix_lo = 0, mix_ld = 0, mix_n = 0;
  int64_t acc_lo = 0, acc_ld = 0;
  int64_t out_lo = 0, out_ld = 0;
};
// `segment`: samples per chunk; `row`: samples per forward row (0 = segment),
// longer than `segment` when the chunks are cut shorter than the model's
// training length (zero padded at the row's end).
void launch_gather_chunks(const float* mix_norm, int64_t length, int64_t shift_offset,
                          int64_t max_shift, int segment, int64_t stride, int64_t chunk0,
                          int count, float* out, cudaStream_t s, int row = 0,
                          const DriverWindow* win = nullptr);
void launch_ola_accumulate(const float* chunks, int64_t length, int64_t shift_offset,
                           int64_t max_shift, int segment, int64_t stride, int64_t chunk0,
                           int count, const float* weight, float* acc, int64_t view_lo,
                           int64_t view_hi, cudaStream_t s, int row = 0);
// output samples [t_lo, t_hi) only (t_hi < 0: to the end)
void launch_ola_finish(const float* acc, int64_t length, int64_t shift_offset, int64_t max_shift,
                       int segment, int64_t stride, const float* weight, const float2* norm,
                       float scale, int mode, float* pass, float* stems, cudaStream_t s,
                       int64_t t_lo = 0, int64_t t_hi = -1, const DriverWindow* win = nullptr);

// stats.cu — fixed-order moment reductions. part is (rows * rowlen positions,
// nslots, 2) doubles; stats[row] = (sum, sum of squares) over the row's
// positions and slots, in an order fixed by the position inside the row.
void launch_row_stats_reduce(const double* part, int nslots, int64_t rowlen, int rows,
                             double* stats, cudaStream_t s);
// stats[row] = sum over k < nparts of part[row][k] (2 doubles each), in order.
void launch_sum_partials(const double* part, int nparts, int rows, double* stats, cudaStream_t s);

// multi.cu — acc[r * ld + c] += tail[r * width + c] (rows x width), the
// boundary merge of the multi-GPU track driver.
void launch_tail_add(float* acc, int64_t ld, const float* tail, int64_t width, int rows,
                     cudaStream_t s);
// dst (rows, width; row stride dld) = src, or += src with `add` (each sum
// rounded on its own); src may be a peer GPU's memory mapped into this process.
void launch_rows(bool add, float* dst, int64_t dld, const float* src, int64_t sld, int rows,
                 int64_t width, cudaStream_t s);

// selftest.cu — one warp waits on a device flag nothing sets and, after
// limit_ns, stores `code` into err and returns (the bounded-wait error path).
void launch_selftest_wait(uint64_t limit_ns, int code, int* err, cudaStream_t s);

// bag.cu — the bag's per-source weighted combination (api.rs:319-361).
// For source s: out = (sum over j < count[s] of out[net[s][j]] * weight[s][j])
// / total[s], or zeros when count[s] == 0. Every out[] buffer and `out` is
// (segments, sources, channels, samples) on the launching device.
constexpr int kBagMaxNets = 8;
constexpr int kBagMaxSources = 4;
struct BagTerms {
  const float* out[kBagMaxNets];
  int net[kBagMaxSources][kBagMaxNets];
  float weight[kBagMaxSources][kBagMaxNets];
  int count[kBagMaxSources];
  float total[kBagMaxSources];
  int sources, channels;
};
void launch_bag_combine(const BagTerms& t, int64_t segments, int64_t samples, float* out,
                        cudaStream_t s);

}  // namespace dmx
