// Tensor-core (tcgen05 / TMEM / TMA) implicit-GEMM convolution for sm_100a.
//
// Persistent: one CTA per SM walks the 128 x BN output tiles (column tiles
// fastest) with cta_group::1 UMMA (kind::tf32, fp32 accumulate in TMEM, two
// accumulators). Warp 0 issues TMA tile loads into a STAGES-deep shared-memory
// ring, warps 2-5 round each landed A tile to nearest tf32, warp 1 issues the
// MMAs (one elected thread), and warps 6-9 drain the previous tile's
// accumulator with tcgen05.ld and apply the same fused epilogues as the SIMT
// path (conv_gemm.cuh) while the next tile's MMAs run. The A operand is an activation tile read
// straight from the channels-last tensor by TMA — the convolution taps are
// coordinate offsets and the padding is TMA's out-of-bounds zero fill, so no
// patch matrix exists anywhere. No load uses cluster multicast.
#pragma once

#include <cuda.h>

#include "conv_gemm.cuh"

namespace dmx {

enum TcAMode : int {
  TC_ROWS = 0,  // A is a [rows][K] matrix; tile = 128 consecutive rows
  TC_2D = 1,    // A is a (B, H, W, C) tensor; tile = 8 x 16 positions; taps (dy, dx)
  TC_1D = 2     // A is a (B, W, C) tensor; tile = 128 positions along W; taps dx
};

struct TcParams {
  int mode;
  int B, Hq, Wq;     // output-position grid (TC_2D) ; rows = B*Hq*Wq (TC_ROWS: B=1,Hq=1)
  int Cin;           // channels per tap (K tile never straddles taps)
  int sy, sx;        // tap stride along H (TC_2D) / W (TC_1D): 1 or 4; input = s*out + d
  int ntaps;
  int dy[kMaxTaps], dx[kMaxTaps];
  int K, Kpad, N, Npad;
  const float* bias;
  // output addressing and epilogue, as in ConvParams
  float* out;
  int64_t o_bs, o_ys, o_xs, o_off;
  double* epi_stats;   // row moments (sum, sum of squares) per statistic row of epi_rowlen positions
  int epi_rowlen;
  double* epi_rowpart;  // scratch: positions x tc_gemm_stat_slots(N) partials (2 doubles each)
  int epi_nslots;
  const float* epi_gamma;
  const float* epi_res;
  const float* epi_emb;
  const float* epi_add;
  int round_out;  // round stored values to nearest tf32 (the output feeds only tf32 GEMMs)
  float* vt_out;  // EPI_STORE: V^T copy of columns >= vt_col0 (see ConvParams)
  int vt_col0, vt_ntok;
  int vt16;       // vt_out holds bf16 values (the bf16 attention's V^T)
  int o_lim, o_lim_ch;  // as in ConvParams
  int a_rounded;  // A holds tf32-rounded values: the MMA reads the TMA tile as landed
  int bf16;       // kind::f16: A is a bf16 activation matrix (TC_ROWS), wk the bf16 weight copy
  uint16_t* out16;  // EPI_STORE / EPI_GELU: store bf16 values here instead of `out`
  int o_pcols;          // as in ConvParams: column groups stored o_pstride apart (0 = off)
  int64_t o_pstride;
  // EPI_DCONV_TAIL: row moments of the GLU input (sum, sum of squares per
  // row of epi_rowlen positions, count values each), GroupNorm weight/bias in
  // the reference's order (value c, gate c + epi_half)
  const double* epi_nstats;
  double epi_count;
  const float* epi_gw;
  const float* epi_gb;
  int epi_half;
  // A transform in the converter (TC_ROWS): a = GELU(GroupNorm(a)) with row
  // moments a_stats (rows of a_rowlen positions, a_count values) and per-
  // channel a_gw / a_gb for channels < a_nvalid; channels >= a_nvalid are 0
  const double* a_stats;
  int a_rowlen, a_nvalid;
  double a_count;
  const float* a_gw;
  const float* a_gb;
  int* err;  // set non-zero when a bounded wait gives up
  int mtiles, ntiles;  // tile space (filled in by launch_tc_gemm)
};

// Host: build the two tensor maps and launch. `a` describes the A operand
// tensor (channels-last, element strides), `w` the K-major packed weights
// [Npad][Kpad]. Returns false when the shape is not supported by the
// tensor-core path (the caller then uses the SIMT kernel).
struct TcOperandA {
  const float* ptr;
  int B, H, W, C;           // TC_2D: (B, H, W, C); TC_1D: (B, W, C); TC_ROWS: rows = W, K = C
  int64_t sb, sh, sw;       // element strides of b, h, w (channels contiguous)
};
bool tc_gemm_supported(const TcOperandA& a, const TcParams& p);
// Partials per output position of the row-moment epilogues (two per column tile).
int tc_gemm_stat_slots(int N);
// wk: K-major weights rounded to nearest tf32 (or, with p.bf16, their bf16
// copy [Npad][Kpad]); wk_lo: their residuals (w - tf32(w)) for the 3xTF32
// split, or null.
void launch_tc_gemm(const TcOperandA& a, const float* wk, const float* wk_lo, const TcParams& p,
                    int epi, cudaStream_t s);

// Tensor-core flash attention (attention_tc.cu). Returns false when the shape
// is not supported (the caller then uses the SIMT kernel).
// vt: V^T as (segment, head, dim, key), written by the projection epilogue.
// out16: store the output as bf16 there instead of `out` (row pitch ldo elements).
// bf16_in: q, kv and vt hold bf16 values (pitches still in elements); both
// products then run on kind::f16.
bool launch_attention_tc(const float* q, int ldq, int q_col, const float* kv, int ldkv, int k_col,
                         int v_col, const float* vt, float* out, int ldo, int B, int heads, int nq,
                         int nk, float scale, int* err, cudaStream_t s, uint16_t* out16 = nullptr,
                         bool bf16_in = false);

}  // namespace dmx
