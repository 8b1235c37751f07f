// Implicit-GEMM convolution: one kernel family for every convolution and
// linear of the HTDemucs v4 forward, over channels-last activations.
//
//   out[p, n] = epilogue( sum_{tap, ci} W[tap*Cin + ci, n] * A(p, tap, ci) )
//
// p runs over an output grid (b, y, x); the input position of a tap is
// (y*sy + dy[tap], x*sx + dx[tap]) and reads zero outside the input (this is
// the padding of every Conv1d/Conv2d, the right-pad of the waveform encoder
// and the zero rows of the transposed convolutions). No im2col matrix is ever
// materialised: the gather happens while the tile is staged in shared memory.
#pragma once

#include "common.cuh"

namespace dmx {

constexpr int kMaxTaps = 16;

enum ProMode : int {
  PRO_NONE = 0,
  PRO_BATCH_AFFINE = 1,  // (v - shift[b]) * scale[b]   (input normalisation)
  PRO_ADD = 2            // v + x2                      (decoder skip connection)
};

enum EpiMode : int {
  EPI_STORE = 0,          // acc + bias
  EPI_GELU = 1,           // gelu(acc + bias)
  EPI_GLU = 2,            // value * sigmoid(gate), columns interleaved (2c, 2c+1)
  EPI_GLU_EMB = 3,        // GLU + emb[y, c]
  EPI_RESIDUAL = 4,       // out = res + gamma[n] * (acc + bias) [+ row moments]
  // tensor-core path only (the DConv branch as GEMMs, see dmx_handle::run_dconv):
  EPI_STORE_STATS = 5,    // store acc + bias and accumulate its row moments
  EPI_STATS = 6,          // row moments of acc + bias, nothing stored
  EPI_DCONV_TAIL = 7      // out[c] = res[c] + gamma[c] * GLU(GroupNorm(acc + bias))
};

struct ConvParams {
  // input gather, element strides: b*i_bs + iy*i_ys + ix*i_xs + ci*i_cs
  const float* x;
  const float* x2;
  int64_t i_bs, i_ys, i_xs, i_cs;
  int Hin, Win, Cin;
  int sy, sx;
  int ntaps;
  int dy[kMaxTaps], dx[kMaxTaps];
  // output grid, M = B * Hq * Wq positions
  int B, Hq, Wq;
  // packed weights [Kpad][Npad] (zero padded), bias [Npad]
  const float* w;
  int K, Npad;
  const float* bias;
  int N;  // live GEMM columns (2C for the GLU modes)
  // output element = b*o_bs + y*o_ys + x*o_xs + o_off + column (GLU modes:
  // column/2); channels are contiguous
  float* out;
  int64_t o_bs, o_ys, o_xs, o_off;
  // prologue
  const float* pro_scale;  // PRO_BATCH_AFFINE: float4 {mean, scale, ..} per segment
  // epilogue
  double* epi_stats;  // EPI_RESIDUAL: per-row (sum, sum of squares) of the output
  int epi_rowlen;
  // scratch of the row moments: one partial (2 doubles) per output position and
  // column tile (conv_gemm_stat_slots(N) of them; the tensor-core kernel needs
  // tc_gemm_stat_slots(N)), reduced in a fixed order after the launch
  double* epi_rowpart;
  const float* epi_gamma;
  const float* epi_res;
  const float* epi_emb;
  const float* epi_add;  // EPI_STORE / EPI_GELU: + add[element] after the activation
  int round_out;         // EPI_STORE: round stored values to nearest tf32
  // EPI_STORE: columns >= vt_col0 are also written transposed per segment and
  // 64-wide head, vt[((b*heads + h)*64 + d)*vt_ntok + token] (attention's V^T)
  float* vt_out;
  int vt_col0, vt_ntok;
  int vt16;  // vt_out holds bf16 values (the tensor-core kernel only)
  // o_lim > 0: output position x (along W) holds groups of o_lim_ch columns
  // for positions 4x, 4x+1, ...; columns of positions >= o_lim are not stored
  int o_lim, o_lim_ch;
  int a_rounded;  // tensor-core path: A already holds tf32-rounded values (no converter pass)
  // tensor-core path, BF16 build: A is a bf16 matrix (x points at uint16 values,
  // row pitch i_xs elements), the GEMM runs kind::f16 on the layer's bf16 weights
  int a_bf16;
  uint16_t* out16;  // EPI_STORE / EPI_GELU: bf16 output instead of `out` (same element offsets)
  // tensor-core path, EPI_STORE / EPI_GELU: o_pcols > 0 splits the columns into
  // groups of o_pcols (a multiple of 16) stored o_pstride elements apart —
  // column g * o_pcols + c goes to element row + g * o_pstride + c (the four
  // output phases of a stride-4 ConvTranspose landing on rows 4 f + phase)
  int o_pcols;
  int64_t o_pstride;
};

void launch_conv_gemm(const ConvParams& p, int pro, int epi, cudaStream_t stream);
int conv_gemm_stat_slots(int N);
// The first encoder convolutions (Cin 2/4, 8 taps, 48 GELU outputs, normalised
// input, dense channels-last output; first_conv.cu). w_host: [K][48] weights
// then the 48 biases, in host memory. False: not that shape.
bool launch_first_conv(const ConvParams& p, int pro, int epi, const float* w_host,
                       cudaStream_t stream);

}  // namespace dmx
