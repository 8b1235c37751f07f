// The segment forward on the device: the handle's launch helpers (one GEMM
// launch picks the tensor-core, first-convolution or SIMT kernel), the DConv
// branch, the transformer layers and the whole HTDemucs v4 launch sequence
// (Htdemucs::forward, host.rs:202-520), plus the workspace sizing and the
// device error flag.
#include <cmath>
#include <cstdio>

#include "runtime.cuh"

using namespace dmx;

void dmx_handle::gemm(const ConvParams& p0, int pro, int epi, const char* tag,
                      const Packed* pk) {
  ConvParams p = p0;
  if (p.epi_stats && !p.epi_rowpart) {
    // scratch of the row moments, sized for either kernel's partials
    const int64_t M = (int64_t)p.B * p.Hq * p.Wq;
    const int slots = std::max(tc_gemm_stat_slots(p.N), conv_gemm_stat_slots(p.N));
    p.epi_rowpart = dalloc((size_t)M * slots * 2);
  }
  ++launches;
  if (p.epi_stats && epi == EPI_RESIDUAL) ++launches;  // the ordered reduction of the moments
  if (!live()) return;
  if (epi == EPI_RESIDUAL && p.epi_stats &&
      p.epi_rowlen < 128)
    throw Error(DMX_ERR_INVALID, "row statistics need rows of at least 128 positions");
  if (stage_timing) {
    const double M = (double)p.B * p.Hq * p.Wq;
    const int cin = pk ? pk->cin_real : p.Cin;
    const double K = (double)p.ntaps * cin;
    const bool glu = epi == EPI_GLU || epi == EPI_GLU_EMB;
    const double nout = glu ? p.N / 2 : p.N;
    double bytes = 4.0 * ((double)p.B * p.Hin * p.Win * cin + K * p.N);
    if (pro == PRO_ADD) bytes += 4.0 * p.B * p.Hin * p.Win * cin;
    bytes += 4.0 * M * nout;
    if (epi == EPI_RESIDUAL) bytes += 4.0 * M * nout;
    mark(tag, 2.0 * M * K * p.N * (pk ? pk->flop_scale : 1.0), bytes);
  }
  if (pk && (cfg.precision == DMX_TF32 || cfg.precision == DMX_TF32X3 || cfg.precision == DMX_BF16) &&
      try_tc(p, pro, epi, *pk))
    return;
  if (p.a_bf16 || p.out16)
    throw Error(DMX_ERR_INVALID, std::string(tag) + ": bf16 operands need the tensor-core kernel");
  if (pk && !pk->host_w.empty() && launch_first_conv(p, pro, epi, pk->host_w.data(), stream))
    return;
  launch_conv_gemm(p, pro, epi, stream);
}

// The tensor-core path alone, for launches the SIMT kernel cannot express
// (split output columns): false, with nothing launched, when the
// tensor-core kernel does not take it; the caller then issues another form.
bool dmx_handle::gemm_tc(const ConvParams& p, int epi, const char* tag, const Packed& pk) {
  if (cfg.precision != DMX_TF32 && cfg.precision != DMX_TF32X3 && cfg.precision != DMX_BF16)
    return false;
  if (epi != EPI_STORE && epi != EPI_GELU) return false;
  if (p.o_pcols % 16 != 0 || p.o_lim != 0 || p.vt_out) return false;
  if (!live()) {
    ++launches;
    return true;
  }
  TcOperandA a;
  TcParams t;
  if (!build_tc(p, pk, a, t)) return false;
  ++launches;
  if (stage_timing) {
    const double M = (double)p.B * p.Hq * p.Wq;
    const double K = (double)p.ntaps * pk.cin_real;
    double bytes = 4.0 * ((double)p.B * p.Hin * p.Win * pk.cin_real + K * p.N) + 4.0 * M * p.N;
    if (p.epi_add) bytes += 4.0 * M * p.N;
    mark(tag, 2.0 * M * K * p.N * pk.flop_scale, bytes);
  }
  launch_tc_gemm(a, wdev + pk.tc_off, cfg.precision == DMX_TF32X3 ? wdev + pk.tc_lo_off : nullptr,
                 t, epi, stream);
  ++tc_launches;
  return true;
}

// The tensor-core path takes a launch when its A operand is a plain
// channels-last tile read (no prologue transform) with stride-1 taps (or
// the strided encoder taps).
bool dmx_handle::try_tc(const ConvParams& p, int pro, int epi, const Packed& pk) {
  if (pro != PRO_NONE || !pk.has_tc || p.i_cs != 1) return false;
  if (epi != EPI_STORE && epi != EPI_GELU && epi != EPI_GLU && epi != EPI_GLU_EMB &&
      epi != EPI_RESIDUAL)
    return false;
  TcOperandA a;
  TcParams t;
  if (!build_tc(p, pk, a, t)) return false;
  // BF16 build: the layers with a bf16 weight copy (the transformer linears) run
  // kind::f16; everything else single-pass tf32 as in the TF32 build
  const float* wk = t.bf16 ? wdev + pk.bf_off : wdev + pk.tc_off;
  launch_tc_gemm(a, wk, cfg.precision == DMX_TF32X3 ? wdev + pk.tc_lo_off : nullptr, t, epi,
                 stream);
  ++tc_launches;
  return true;
}

// ConvParams -> tensor-core operand and parameters; false when unsupported.
bool dmx_handle::build_tc(const ConvParams& p, const Packed& pk, TcOperandA& a, TcParams& t) {
  if (!pk.has_tc || p.i_cs != 1) return false;
  std::memset(&t, 0, sizeof(t));
  a.ptr = p.x;
  a.C = p.Cin;
  bool taps_zero = true;
  for (int i = 0; i < p.ntaps; ++i) taps_zero = taps_zero && p.dy[i] == 0 && p.dx[i] == 0;
  const bool rows = taps_zero && p.Hq == p.Hin && p.Wq == p.Win && p.i_xs == p.Cin &&
                    p.i_ys == (int64_t)p.Win * p.Cin && p.i_bs == (int64_t)p.Hin * p.Win * p.Cin;
  if (rows) {
    t.mode = TC_ROWS;
    a.B = 1;
    a.H = 1;
    a.W = p.B * p.Hin * p.Win;
    a.sw = p.Cin;
    a.sh = a.sb = 0;
  } else if (p.Hin == 1 && p.Hq == 1) {
    t.mode = TC_1D;
    a.B = p.B;
    a.H = 1;
    a.W = p.Win;
    a.sw = p.i_xs;
    a.sh = 0;
    a.sb = p.i_bs;
  } else {
    t.mode = TC_2D;
    a.B = p.B;
    a.H = p.Hin;
    a.W = p.Win;
    a.sw = p.i_xs;
    a.sh = p.i_ys;
    a.sb = p.i_bs;
  }
  t.B = p.B;
  t.Hq = p.Hq;
  t.Wq = p.Wq;
  t.Cin = p.Cin;
  t.sy = p.sy;
  t.sx = p.sx;
  t.ntaps = p.ntaps;
  for (int i = 0; i < p.ntaps; ++i) {
    t.dy[i] = p.dy[i];
    t.dx[i] = p.dx[i];
  }
  t.K = p.K;
  t.Kpad = pk.K;
  t.N = p.N;
  t.Npad = p.Npad;
  t.bias = p.bias;
  t.out = p.out;
  t.o_bs = p.o_bs;
  t.o_ys = p.o_ys;
  t.o_xs = p.o_xs;
  t.o_off = p.o_off;
  t.epi_stats = p.epi_stats;
  t.epi_rowlen = p.epi_rowlen;
  t.epi_rowpart = p.epi_rowpart;
  t.epi_nslots = tc_gemm_stat_slots(p.N);
  t.epi_gamma = p.epi_gamma;
  t.epi_res = p.epi_res;
  t.epi_emb = p.epi_emb;
  t.epi_add = p.epi_add;
  t.round_out = p.round_out;
  t.vt_out = p.vt_out;
  t.vt_col0 = p.vt_col0;
  t.vt_ntok = p.vt_ntok;
  t.vt16 = p.vt16;
  t.o_lim = p.o_lim;
  t.o_lim_ch = p.o_lim_ch;
  t.a_rounded = p.a_rounded;
  t.o_pcols = p.o_pcols;
  t.o_pstride = p.o_pstride;
  t.err = err;
  t.bf16 = p.a_bf16;
  t.out16 = p.out16;
  if (t.bf16 && !pk.has_bf) return false;
  return tc_gemm_supported(a, t);
}

namespace dmx {

namespace {

ConvParams base_params(const Packed& pk, const float* W0) {
  ConvParams p;
  std::memset(&p, 0, sizeof(p));
  p.w = W0 + pk.w_off;
  p.bias = W0 + pk.b_off;
  p.K = pk.K;
  p.Npad = pk.Npad;
  p.N = pk.N;
  p.ntaps = (int)pk.taps.size();
  for (int i = 0; i < p.ntaps; ++i) {
    p.dy[i] = pk.taps[i].dy;
    p.dx[i] = pk.taps[i].dx;
  }
  p.sy = p.sx = 1;
  return p;
}

// Channels-last activation geometry: (B, H, W, C).
void set_input(ConvParams& p, const float* x, int B, int H, int W, int C) {
  (void)B;
  p.x = x;
  p.Hin = H;
  p.Win = W;
  p.Cin = C;
  p.i_cs = 1;
  p.i_xs = C;
  p.i_ys = (int64_t)W * C;
  p.i_bs = (int64_t)H * W * C;
}
void set_output(ConvParams& p, float* out, int B, int Hq, int Wq, int Cout) {
  p.B = B;
  p.Hq = Hq;
  p.Wq = Wq;
  p.out = out;
  p.o_xs = Cout;
  p.o_ys = (int64_t)Wq * Cout;
  p.o_bs = (int64_t)Hq * Wq * Cout;
  p.o_off = 0;
}

// DConv residual branch in place on x (rows, T, C) channels-last
// (host.rs:985-1059): per layer one fused launch for rows of at most one tile
// (the spectral branch), three tiled launches for longer rows (the waveform
// branch); the kernels are in dconv.cu.
// One tensor-core GEMM of the DConv branch, always split 3xTF32 (the branch
// stays fp32-accurate in every build); `ext` supplies the A transform and the
// DConv epilogue fields.
// The BF16 build runs the DConv contractions single-pass tf32 (the TF32 and
// TF32X3 builds keep 3xTF32): at the benchmark's weights the branch's
// LayerScale (1e-4) scales its error down with its output.
bool dconv_single_pass(const dmx_handle* h) { return h->cfg.precision == DMX_BF16; }

void dconv_gemm(dmx_handle* h, const ConvParams& p, int epi, const Packed& pk, const TcParams& ext) {
  TcOperandA a;
  TcParams t;
  if (!h->build_tc(p, pk, a, t)) throw Error(DMX_ERR_INVALID, "dconv: tensor-core shape unsupported");
  t.epi_nstats = ext.epi_nstats;
  t.epi_count = ext.epi_count;
  t.epi_gw = ext.epi_gw;
  t.epi_gb = ext.epi_gb;
  t.epi_half = ext.epi_half;
  t.a_stats = ext.a_stats;
  t.a_rowlen = ext.a_rowlen;
  t.a_nvalid = ext.a_nvalid;
  t.a_count = ext.a_count;
  t.a_gw = ext.a_gw;
  t.a_gb = ext.a_gb;
  launch_tc_gemm(a, h->W(pk.tc_off), dconv_single_pass(h) ? nullptr : h->W(pk.tc_lo_off), t, epi,
                 h->stream);
  ++h->tc_launches;
}

// The DConv branch as two persistent tensor-core GEMMs per layer around a
// SIMT pass, for rows of any length: conv1 (taps as TMA offsets) storing y
// and its row moments; the row moments of z from g = GELU(GroupNorm1(y)) by
// the quadratic form (dconv.cu); conv2 with GELU(GroupNorm1(y)) applied to
// each A tile by the converter warps and a GroupNorm2 + GLU + LayerScale +
// residual epilogue into x. Moments are f64 partials per position (conv1) or
// per block (z), added in a fixed order per row.
void run_dconv_gemm(dmx_handle* h, const DConvFull& dc, float* x, int rows, int T,
                    bool round_out) {
  const int C = dc.C, hid = dc.hidden;
  const int64_t positions = (int64_t)rows * T;
  const int kg = dc.layer[0].conv2.K;  // y row width = conv2's padded K
  float* y = h->falloc((size_t)positions * kg);
  double* st = h->dalloc((size_t)rows * 4);
  double* ypart = h->dalloc((size_t)positions * tc_gemm_stat_slots(dc.layer[0].conv1.N) * 2);
  double* zpart = h->dalloc((size_t)rows * dconv_zstats_parts(T) * 2);
  for (int d = 0; d < 2; ++d) {
    const DConvLayerW& L = dc.layer[d];
    h->mark("dconv.gemm" + std::to_string(C), 10.0 * positions * C * hid, 8.0 * positions * C);
    h->launches += 5;
    if (!h->live()) continue;
    TcParams ext;
    std::memset(&ext, 0, sizeof(ext));
    {  // conv1: x (rows, T, C) -> y (rows, T, kg), the first hid columns
      ConvParams p = base_params(L.conv1, h->wdev);
      set_input(p, x, rows, 1, T, C);
      set_output(p, y, rows, 1, T, kg);
      p.epi_stats = st;
      p.epi_rowlen = T;
      p.epi_rowpart = ypart;
      dconv_gemm(h, p, EPI_STORE_STATS, L.conv1, ext);
    }
    ConvParams q = base_params(L.conv2, h->wdev);
    set_input(q, y, 1, 1, (int)positions, kg);
    set_output(q, x, 1, 1, (int)positions, C);
    q.epi_rowlen = T;
    ext.a_stats = st;
    ext.a_rowlen = T;
    ext.a_nvalid = hid;
    ext.a_count = (double)hid * T;
    ext.a_gw = h->W(L.n1w.off);
    ext.a_gb = h->W(L.n1b.off);
    // moments of z from g alone (v.g~, g~'Mg~), without a conv2 pass
    if (!launch_dconv_zstats(C, y, kg, rows, T, h->W(L.n1w.off), h->W(L.n1b.off), st, st + 2 * rows,
                             zpart, h->W(L.zq_off), h->stream))
      throw Error(DMX_ERR_INVALID, "dconv: moments of z for this width");
    q.epi_stats = nullptr;  // the output
    ext.epi_nstats = st + 2 * rows;
    ext.epi_count = 2.0 * C * T;
    ext.epi_gw = h->W(L.n2w.off);
    ext.epi_gb = h->W(L.n2b.off);
    ext.epi_half = C;
    q.epi_gamma = h->W(L.gamma.off);
    q.epi_res = x;
    q.round_out = round_out && d == 1;
    dconv_gemm(h, q, EPI_DCONV_TAIL, L.conv2, ext);
    h->after("dconv");
  }
}

// The narrowest DConv width that runs as the three tensor-core GEMMs of
// run_dconv_gemm when the fused kernel does not take it.
#ifndef DMX_DCONV_GEMM_MIN_C
#define DMX_DCONV_GEMM_MIN_C 384
#endif

// round_out: the branch's output feeds only a tf32 GEMM (the TF32 build): the
// last layer stores it rounded to nearest tf32 so that GEMM needs no converter.
void run_dconv(dmx_handle* h, const DConvFull& dc, float* x, int rows, int T, bool round_out) {
  const int C = dc.C, hid = dc.hidden;
  const int64_t positions = (int64_t)rows * T;
  const bool tf32 = h->cfg.precision == DMX_TF32 || h->cfg.precision == DMX_TF32X3 ||
                    h->cfg.precision == DMX_BF16;
  const bool has_tc = dc.layer[0].conv1.has_tc && dc.layer[0].conv2.has_tc;
  // TF32 builds: tensor cores (3xTF32, fp32-accurate) for the narrow layers
  // (the fused kernel: one launch per spectral row, three over the tiles of a
  // waveform row) and the widest layers (three GEMMs, where the SIMT kernels
  // are compute-bound); the SIMT kernels are faster elsewhere. The BF16
  // build's single-pass contractions also take C 192 onto a fused kernel.
  const bool tc = tf32 && has_tc && !dc.layer[0].zq.empty() &&
                  dconv_tc_supported(C, T, dconv_single_pass(h));
  if (tf32 && has_tc && !tc && C >= DMX_DCONV_GEMM_MIN_C) {
    run_dconv_gemm(h, dc, x, rows, T, round_out);
    return;
  }
  const int tiles = tc ? dconv_tc_tiles(T) : dconv_tiles(T);
  const bool fused = tc ? tiles == 1 : dconv_row_fused(T);
  float* y = fused ? nullptr : h->falloc((size_t)positions * (tc ? dconv_tc_ystride(C) : hid));
  double* part = fused ? nullptr : h->dalloc((size_t)rows * tiles * 4);
  for (int d = 0; d < 2; ++d) {
    const DConvLayerW& L = dc.layer[d];
    DConvArgs a;
    std::memset(&a, 0, sizeof(a));
    a.x = x;
    a.C = C;
    a.rows = rows;
    a.T = T;
    a.dil = 1 << d;
    a.tiles = tiles;
    a.w1 = h->W(L.conv1.w_off);
    a.w1_ld = L.conv1.Npad;
    a.b1 = h->W(L.conv1.b_off);
    a.n1w = h->W(L.n1w.off);
    a.n1b = h->W(L.n1b.off);
    a.w2 = h->W(L.conv2.w_off);
    a.w2_ld = L.conv2.Npad;
    a.b2 = h->W(L.conv2.b_off);
    a.n2w = h->W(L.n2w.off);
    a.n2b = h->W(L.n2b.off);
    a.gamma = h->W(L.gamma.off);
    a.y = y;
    a.part1 = part;
    a.part2 = part ? part + 2 * (size_t)rows * tiles : nullptr;
    a.err = h->err;
    a.round_out = round_out && d == 1;
    a.single = dconv_single_pass(h);
    a.w1_tc = h->W(L.conv1.tc_off);
    a.w1_tc_lo = h->W(L.conv1.tc_lo_off);
    a.w1_npad = L.conv1.Npad;
    a.w2_tc = h->W(L.conv2.tc_off);
    a.w2_tc_lo = h->W(L.conv2.tc_lo_off);
    a.w2_npad = L.conv2.Npad;
    a.zq_host = L.zq.empty() ? nullptr : L.zq.data();
    a.zq_dev = h->W(L.zq_off);
    // algorithmic work: conv1 (3C -> hid) + conv2 (hid -> 2C) per position;
    // x read once and written once
    h->mark(std::string(tc ? (fused ? "dconv.tc" : "dconv.tctiled")
                           : (fused ? "dconv.row" : "dconv.tiled")) +
                std::to_string(C),
            10.0 * positions * C * hid, 8.0 * positions * C);
    if (h->live()) {
      if (!(tc ? launch_dconv_tc(a, h->stream) : launch_dconv(a, h->stream)))
        throw Error(DMX_ERR_INVALID, "dconv: unsupported shape");
      h->after("dconv");
    }
    h->launches += fused ? 1 : 3;
  }
}

// Host-side tracing: copy a device tensor and hand it over in the reference's
// layout. kind 0: freq (B, F, T, C) -> (B, C, F, T); kind 1: time (B, T, C)
// -> (B, C, T); kind 2: as is with the given shape; kind 3: frame-major freq
// (B, T, F, C) -> (B, C, F, T), dims given as {B, F, T, C}.
void trace_tensor(dmx_handle* h, const std::string& name, const float* dev, int kind,
                  std::vector<int64_t> dims, const float* minus = nullptr) {
  if (!h->trace || h->measuring) return;
  size_t n = 1;
  for (int64_t d : dims) n *= (size_t)d;
  std::vector<float> host(n), out(n);
  CK(cudaStreamSynchronize(h->stream));
  CK(cudaMemcpy(host.data(), dev, n * sizeof(float), cudaMemcpyDeviceToHost));
  if (minus) {  // the stored tensor already carries the next layer's skip connection
    std::vector<float> sub(n);
    CK(cudaMemcpy(sub.data(), minus, n * sizeof(float), cudaMemcpyDeviceToHost));
    for (size_t i = 0; i < n; ++i) host[i] -= sub[i];
  }
  std::vector<int64_t> shape;
  if (kind == 0) {
    const int64_t B = dims[0], F = dims[1], T = dims[2], C = dims[3];
    for (int64_t b = 0; b < B; ++b)
      for (int64_t f = 0; f < F; ++f)
        for (int64_t t = 0; t < T; ++t)
          for (int64_t c = 0; c < C; ++c)
            out[((b * C + c) * F + f) * T + t] = host[((b * F + f) * T + t) * C + c];
    shape = {B, C, F, T};
  } else if (kind == 3) {
    const int64_t B = dims[0], F = dims[1], T = dims[2], C = dims[3];
    for (int64_t b = 0; b < B; ++b)
      for (int64_t t = 0; t < T; ++t)
        for (int64_t f = 0; f < F; ++f)
          for (int64_t c = 0; c < C; ++c)
            out[((b * C + c) * F + f) * T + t] = host[((b * T + t) * F + f) * C + c];
    shape = {B, C, F, T};
  } else if (kind == 1) {
    const int64_t B = dims[0], T = dims[1], C = dims[2];
    for (int64_t b = 0; b < B; ++b)
      for (int64_t t = 0; t < T; ++t)
        for (int64_t c = 0; c < C; ++c) out[(b * C + c) * T + t] = host[(b * T + t) * C + c];
    shape = {B, C, T};
  } else {
    out = host;
    shape = dims;
  }
  h->trace(name.c_str(), out.data(), shape.data(), (int)shape.size(), h->trace_user);
}

// One transformer layer on stream X (B, n, 512), in place (host.rs:1315-1429).
struct XfBufs {
  float *xn, *kvn, *qkv, *kv2, *att, *hid;
  float *vt1, *vt2;  // V^T copies for the tensor-core attention
  double* stats;
};

// Transformer linear layers. In the TF32 build every A operand here (the
// LayerNorm outputs, the first FFN layer's GELU output, the attention output)
// is produced already rounded to nearest tf32, so the GEMM skips its converter
// pass; the operands are the same values the converter would produce.
bool xf_rounded(const dmx_handle* h) { return h->cfg.precision == DMX_TF32; }
// The convolution GEMMs run single-pass tf32 in the TF32 and BF16 builds: their
// producers store operands rounded to nearest tf32 the same way.
bool conv_rounded(const dmx_handle* h) {
  return h->cfg.precision == DMX_TF32 || h->cfg.precision == DMX_BF16;
}
// The tensor-core attention (tf32) runs in the TF32 and BF16 builds.
bool tc_attention(const dmx_handle* h) { return conv_rounded(h); }
// BF16 build: the transformer's linears take bf16 A operands, which their
// producers (LayerNorm, the first FFN layer, attention) store as bf16.
bool xf_bf16(const dmx_handle* h) { return h->cfg.precision == DMX_BF16; }
uint16_t* u16(float* p) { return reinterpret_cast<uint16_t*>(p); }

void xf_gemm(dmx_handle* h, const char* tag, const Packed& pk, const float* in, int B, int n,
             float* out, int epi, const float* res = nullptr, const float* gamma = nullptr,
             double* stats = nullptr, bool round_out = false, float* vt = nullptr,
             int vt_col0 = 0, bool out_bf16 = false, bool vt16 = false) {
  ConvParams p = base_params(pk, h->wdev);
  p.round_out = round_out;
  p.a_rounded = xf_rounded(h);
  p.a_bf16 = xf_bf16(h);
  p.out16 = out_bf16 ? u16(out) : nullptr;
  p.vt_out = vt;
  p.vt_col0 = vt_col0;
  p.vt_ntok = n;
  p.vt16 = vt16 ? 1 : 0;
  const int cin = pk.K;
  set_input(p, in, B, 1, n, cin);
  set_output(p, out, B, 1, n, pk.N);
  p.epi_res = res;
  p.epi_gamma = gamma;
  p.epi_stats = stats;
  p.epi_rowlen = n;
  h->gemm(p, PRO_NONE, epi, tag, &pk);
}

void xf_tail(dmx_handle* h, const LayerW& L, float* X, int B, int n, const XfBufs& bb,
             const Vec& nw, const Vec& nb) {
  // out-projection + LayerScale residual
  xf_gemm(h, "xf.outproj", L.out, bb.att, B, n, X, EPI_RESIDUAL, X, h->W(L.g1.off));
  h->mark("xf.layernorm", 0.0, 8.0 * B * n * 512);
  if (h->live())
    launch_layer_norm(X, (int64_t)B * n, n, h->W(nw.off), h->W(nb.off), nullptr, bb.xn, h->stream,
                      xf_rounded(h), xf_bf16(h) ? u16(bb.xn) : nullptr);
  ++h->launches;
  xf_gemm(h, "xf.ffn1", L.lin1, bb.xn, B, n, bb.hid, EPI_GELU, nullptr, nullptr, nullptr,
          xf_rounded(h), nullptr, 0, xf_bf16(h));
  xf_gemm(h, "xf.ffn2", L.lin2, bb.hid, B, n, X, EPI_RESIDUAL, X, h->W(L.g2.off), bb.stats);
  h->mark("xf.groupnorm", 0.0, 8.0 * B * n * 512);
  if (h->live()) launch_group_norm_apply(X, B, n, bb.stats, h->W(L.now.off), h->W(L.nob.off), h->stream);
  ++h->launches;
}

void xf_self(dmx_handle* h, const LayerW& L, float* X, int B, int n, const XfBufs& bb) {
  h->mark("xf.layernorm", 0.0, 8.0 * B * n * 512);
  if (h->live()) launch_layer_norm(X, (int64_t)B * n, n, h->W(L.n1w.off), h->W(L.n1b.off), nullptr, bb.xn,
                                   h->stream, xf_rounded(h), xf_bf16(h) ? u16(bb.xn) : nullptr);
  ++h->launches;
  const bool tc_attn = tc_attention(h);
  const bool bfa = tc_attn && xf_bf16(h);  // q, k, v and V^T stored as bf16 for kind::f16
  xf_gemm(h, "xf.qkv", L.qkv, bb.xn, B, n, bb.qkv, EPI_STORE, nullptr, nullptr, nullptr,
          tc_attn && !bfa, tc_attn ? bb.vt1 : nullptr, 1024, bfa, bfa);
  h->mark("xf.attention", 4.0 * B * n * n * 512, (bfa ? 2.0 : 4.0) * B * n * 512 * 4);
  if (h->live() && !(tc_attn && launch_attention_tc(bb.qkv, 1536, 0, bb.qkv, 1536, 512, 1024, bb.vt1,
                                                     bb.att, 512, B, 8, n, n, 0.125f, h->err,
                                                     h->stream, xf_bf16(h) ? u16(bb.att) : nullptr,
                                                     bfa))) {
    if (xf_bf16(h)) throw Error(DMX_ERR_INVALID, "attention: the bf16 output needs the tensor-core kernel");
    launch_flash_attention(bb.qkv, 1536, bb.qkv + 512, bb.qkv + 1024, 1536, bb.att, 512, B, 8, n, n,
                           0.125f, h->stream);
  }
  ++h->launches;
  xf_tail(h, L, X, B, n, bb, L.n2w, L.n2b);
}

// kv projection of the other stream for a cross layer (LN2 of this layer).
void xf_cross_kv(dmx_handle* h, const LayerW& L, const float* other, int B, int n_other,
                 float* kv_out, float* scratch, float* vt) {
  h->mark("xf.layernorm", 0.0, 8.0 * B * n_other * 512);
  if (h->live())
    launch_layer_norm(other, (int64_t)B * n_other, n_other, h->W(L.n2w.off), h->W(L.n2b.off), nullptr,
                      scratch, h->stream, xf_rounded(h), xf_bf16(h) ? u16(scratch) : nullptr);
  ++h->launches;
  const bool tc_attn = tc_attention(h);
  const bool bfa = tc_attn && xf_bf16(h);
  xf_gemm(h, "xf.kv", L.kv, scratch, B, n_other, kv_out, EPI_STORE, nullptr, nullptr, nullptr,
          tc_attn && !bfa, tc_attn ? vt : nullptr, 512, bfa, bfa);
}

void xf_cross(dmx_handle* h, const LayerW& L, float* X, int B, int n, const float* kv,
              const float* vt, int n_other, const XfBufs& bb) {
  h->mark("xf.layernorm", 0.0, 8.0 * B * n * 512);
  if (h->live()) launch_layer_norm(X, (int64_t)B * n, n, h->W(L.n1w.off), h->W(L.n1b.off), nullptr, bb.xn,
                                   h->stream, xf_rounded(h), xf_bf16(h) ? u16(bb.xn) : nullptr);
  ++h->launches;
  const bool tc_attn = tc_attention(h);
  const bool bfa = tc_attn && xf_bf16(h);
  xf_gemm(h, "xf.q", L.q, bb.xn, B, n, bb.qkv, EPI_STORE, nullptr, nullptr, nullptr,
          tc_attn && !bfa, nullptr, 0, bfa);
  h->mark("xf.attention", 4.0 * B * n * n_other * 512,
          (bfa ? 2.0 : 4.0) * B * (2.0 * n + 2.0 * n_other) * 512);
  if (h->live() && !(tc_attn && launch_attention_tc(bb.qkv, 512, 0, kv, 1024, 0, 512, vt, bb.att,
                                                     512, B, 8, n, n_other, 0.125f, h->err,
                                                     h->stream, xf_bf16(h) ? u16(bb.att) : nullptr,
                                                     bfa))) {
    if (xf_bf16(h)) throw Error(DMX_ERR_INVALID, "attention: the bf16 output needs the tensor-core kernel");
    launch_flash_attention(bb.qkv, 512, kv, kv + 512, 1024, bb.att, 512, B, 8, n, n_other, 0.125f,
                           h->stream);
  }
  ++h->launches;
  xf_tail(h, L, X, B, n, bb, L.n3w, L.n3b);
}

}  // namespace

void forward(dmx_handle* h, const float* mix, int G, float* out) {
  const int L = kSegment;
  const Model& m = h->m;
  h->ws_off = 0;
  cudaStream_t s = h->stream;
  const float2* tw = reinterpret_cast<const float2*>(h->W(m.tw_off));

  // (a) spectrogram + moments (per-segment partials, added in a fixed order)
  double* part_f = h->dalloc((size_t)G * kFrames * 2);
  double* part_t = h->dalloc((size_t)G * kWaveMomentBlocks * 2);
  float4* norm = static_cast<float4*>(h->alloc((size_t)G * 2 * sizeof(float4)));
  float4* norm_f = norm;
  float4* norm_t = norm + G;
  float* X = h->falloc((size_t)G * kBins * kFrames * 4);
  h->mark("spec.stft", 0.0, 4.0 * G * (2.0 * L + (double)kBins * kFrames * 4));
  if (h->live()) {
    launch_stft_cac(mix, G, h->W(m.window.off), tw, X, part_f, s);
    launch_wave_moments(mix, G, 2LL * L, part_t, s);
    launch_norm_finalize(part_f, kFrames, (double)kBins * kFrames * 4, G, norm_f, s);
    launch_norm_finalize(part_t, kWaveMomentBlocks, 2.0 * L, G, norm_t, s);
    h->after("spectrogram");
  }
  h->launches += 4;

  // (b) encoders
  float* skip[4];
  float* tskip[4];
  int Fs[5], Cs[5], Ts[5], TCs[5], lengths_t[4];
  Fs[0] = kBins;
  Cs[0] = 4;
  Ts[0] = L;
  TCs[0] = 2;
  const float* xin = X;
  const float* tin = mix;
  for (int i = 0; i < 4; ++i) {
    // time encoder (host.rs:625-678)
    {
      const EncW& E = m.tenc[i];
      const int Tin = Ts[i];
      lengths_t[i] = Tin;
      const int Tpad = (Tin + 3) / 4 * 4;
      const int To = (Tpad + 4 - 8) / 4 + 1;
      const int Co = E.cout;
      float* y = h->falloc((size_t)G * To * Co);
      ConvParams p = base_params(E.conv, h->wdev);
      if (i == 0) {  // raw (G, 2, L) waveform, normalised on load
        p.x = tin;
        p.Hin = 1;
        p.Win = L;
        p.Cin = 2;
        p.i_cs = L;
        p.i_xs = 1;
        p.i_ys = 0;
        p.i_bs = 2LL * L;
        p.pro_scale = reinterpret_cast<const float*>(norm_t);
      } else {
        set_input(p, tin, G, 1, Tin, TCs[i]);
      }
      p.sx = 4;
      set_output(p, y, G, 1, To, Co);
      h->gemm(p, i == 0 ? PRO_BATCH_AFFINE : PRO_NONE, EPI_GELU, ("tenc.conv" + std::to_string(i)).c_str(), &E.conv);
      run_dconv(h, h->tenc_dc[i], y, G, To, conv_rounded(h));
      float* z = h->falloc((size_t)G * To * Co);
      ConvParams r = base_params(E.rewrite, h->wdev);
      set_input(r, y, G, 1, To, Co);
      set_output(r, z, G, 1, To, Co);
      r.a_rounded = conv_rounded(h);  // the DConv output, rounded
      h->gemm(r, PRO_NONE, EPI_GLU, ("tenc.rewrite" + std::to_string(i)).c_str(), &E.rewrite);
      tskip[i] = z;
      tin = z;
      Ts[i + 1] = To;
      TCs[i + 1] = Co;
      trace_tensor(h, "tencoder." + std::to_string(i), z, 1, {G, To, Co});
    }
    // freq encoder (host.rs:577-622)
    {
      const EncW& E = m.enc[i];
      const int F = Fs[i], Fo = (F + 4 - 8) / 4 + 1, Co = E.cout;
      float* y = h->falloc((size_t)G * Fo * kFrames * Co);
      ConvParams p = base_params(E.conv, h->wdev);
      set_input(p, xin, G, F, kFrames, Cs[i]);
      p.sy = 4;
      if (i == 0) p.pro_scale = reinterpret_cast<const float*>(norm_f);
      set_output(p, y, G, Fo, kFrames, Co);
      h->gemm(p, i == 0 ? PRO_BATCH_AFFINE : PRO_NONE, EPI_GELU, ("enc.conv" + std::to_string(i)).c_str(), &E.conv);
      run_dconv(h, h->enc_dc[i], y, G * Fo, kFrames, conv_rounded(h));
      float* z = h->falloc((size_t)G * Fo * kFrames * Co);
      ConvParams r = base_params(E.rewrite, h->wdev);
      set_input(r, y, G, Fo, kFrames, Co);
      set_output(r, z, G, Fo, kFrames, Co);
      if (i == 0) r.epi_emb = h->W(m.emb.off);
      r.a_rounded = conv_rounded(h);  // the DConv output, rounded
      h->gemm(r, PRO_NONE, i == 0 ? EPI_GLU_EMB : EPI_GLU, ("enc.rewrite" + std::to_string(i)).c_str(), &E.rewrite);
      skip[i] = z;
      xin = z;
      Fs[i + 1] = Fo;
      Cs[i + 1] = Co;
      trace_tensor(h, i == 0 ? "encoder.0.post_emb" : "encoder." + std::to_string(i), z, 0,
                   {G, Fo, kFrames, Co});
    }
  }

  // (c) channel up-samplers into token layouts (host.rs:320-338, 845-890)
  const int Fb = Fs[4], Tb = kFrames, ntok = Fb * Tb, Tt = Ts[4];
  const int D = 512;
  float* S = h->falloc((size_t)G * ntok * D);
  float* Tk = h->falloc((size_t)G * Tt * D);
  XfBufs bb;
  bb.xn = h->falloc((size_t)G * ntok * D);
  bb.kvn = h->falloc((size_t)G * ntok * D);
  bb.qkv = h->falloc((size_t)G * ntok * 3 * D);
  bb.kv2 = h->falloc((size_t)G * ntok * 2 * D);
  bb.att = h->falloc((size_t)G * ntok * D);
  bb.hid = h->falloc((size_t)G * ntok * 4 * D);
  bb.stats = h->dalloc((size_t)G * 2);
  bb.vt1 = h->falloc((size_t)G * ntok * D);
  bb.vt2 = h->falloc((size_t)G * ntok * D);
  {
    ConvParams p = base_params(m.up, h->wdev);
    set_input(p, skip[3], G, Fb, Tb, Cs[4]);
    p.B = G;
    p.Hq = Fb;
    p.Wq = Tb;
    p.out = bb.kvn;  // tokens t*Fb + f
    p.o_bs = (int64_t)ntok * D;
    p.o_ys = D;
    p.o_xs = (int64_t)Fb * D;
    h->gemm(p, PRO_NONE, EPI_STORE, "xf.upsample", &m.up);
    ConvParams q = base_params(m.up_t, h->wdev);
    set_input(q, tskip[3], G, 1, Tt, TCs[4]);
    set_output(q, bb.kv2, G, 1, Tt, D);
    h->gemm(q, PRO_NONE, EPI_STORE, "xf.upsample", &m.up_t);
    h->mark("xf.layernorm", 0.0, 8.0 * G * (ntok + Tt) * D);
    if (h->live()) {
      launch_layer_norm(bb.kvn, (int64_t)G * ntok, ntok, h->W(m.norm_in_w.off), h->W(m.norm_in_b.off),
                        h->W(m.pos2d.off), S, s);
      launch_layer_norm(bb.kv2, (int64_t)G * Tt, Tt, h->W(m.norm_in_t_w.off), h->W(m.norm_in_t_b.off),
                        h->W(m.pos1d.off), Tk, s);
    }
    h->launches += 2;
    trace_tensor(h, "crosstransformer.in#0", S, 2, {G, ntok, D});
    trace_tensor(h, "crosstransformer.in#1", Tk, 2, {G, Tt, D});
  }
  // (d) five layers, alternating self / cross (host.rs:899-936)
  for (int l = 0; l < 5; ++l) {
    const LayerW& A = m.layers[l];
    const LayerW& At = m.layers_t[l];
    if (!A.cross) {
      xf_self(h, A, S, G, ntok, bb);
      xf_self(h, At, Tk, G, Tt, bb);
    } else {
      // kv for the time stream from the OLD spectral stream, first
      xf_cross_kv(h, At, S, G, ntok, bb.kv2, bb.kvn, bb.vt2);
      float* kv_s = bb.hid;  // spectral layer's kv from the time stream (hid is free here)
      xf_cross_kv(h, A, Tk, G, Tt, kv_s, bb.xn, bb.vt1);
      // the spectral layer needs its kv before xf_tail reuses hid: copy-free
      // ordering — attention consumes kv_s before the FFN writes hid.
      xf_cross(h, A, S, G, ntok, kv_s, bb.vt1, Tt, bb);
      xf_cross(h, At, Tk, G, Tt, bb.kv2, bb.vt2, ntok, bb);
    }
    trace_tensor(h, "crosstransformer.layers." + std::to_string(l), S, 2, {G, ntok, D});
    trace_tensor(h, "crosstransformer.layers_t." + std::to_string(l), Tk, 2, {G, Tt, D});
  }
  // (e) channel down-samplers back to (G, F, T, 384) and (G, T, 384)
  float* x = h->falloc((size_t)G * ntok * Cs[4]);
  float* xt = h->falloc((size_t)G * Tt * TCs[4]);
  {
    ConvParams p = base_params(m.down, h->wdev);
    p.x = S;
    p.Hin = Fb;
    p.Win = Tb;
    p.Cin = D;
    p.i_cs = 1;
    p.i_ys = D;
    p.i_xs = (int64_t)Fb * D;
    p.i_bs = (int64_t)ntok * D;
    set_output(p, x, G, Fb, Tb, Cs[4]);
    p.epi_add = skip[3];
    p.round_out = conv_rounded(h);  // feeds only the first decoder's rewrite
    h->gemm(p, PRO_NONE, EPI_STORE, "xf.downsample", &m.down);
    ConvParams q = base_params(m.down_t, h->wdev);
    set_input(q, Tk, G, 1, Tt, D);
    set_output(q, xt, G, 1, Tt, TCs[4]);
    q.epi_add = tskip[3];
    q.round_out = conv_rounded(h);
    h->gemm(q, PRO_NONE, EPI_STORE, "xf.downsample", &m.down_t);
  }

  // (f) decoders, innermost first (host.rs:408-450)
  int F = Fb, C = Cs[4], Tc = Tt, Ct = TCs[4];
  for (int e = 0; e < 4; ++e) {
    const bool last = e == 3;
    const int j = 3 - e;
    {  // freq decoder (host.rs:682-759)
      const DecW& Dw = m.dec[e];
      float* g = h->falloc((size_t)G * F * kFrames * C);
      ConvParams r = base_params(Dw.rewrite, h->wdev);
      set_input(r, x, G, F, kFrames, C);
      set_output(r, g, G, F, kFrames, C);
      r.a_rounded = conv_rounded(h);  // the down-sampler's or previous decoder's output, rounded
      h->gemm(r, PRO_NONE, EPI_GLU, ("dec.rewrite" + std::to_string(e)).c_str(), &Dw.rewrite);
      run_dconv(h, h->dec_dc[e], g, G * F, kFrames, conv_rounded(h));
      const int Co = Dw.cout, Fo = 4 * F;
      float* o = h->falloc((size_t)G * Fo * kFrames * Co);
      if (last) {
        // the spectrogram for the iSTFT, frame-major (b, t, f, c): one GEMM
        // over the input rows, whose 4 x Co outputs (f = 4 f_in + phase) are
        // contiguous
        ConvParams p = base_params(Dw.convt_all, h->wdev);
        set_input(p, g, G, F, kFrames, C);
        p.B = G;
        p.Hq = F;
        p.Wq = kFrames;
        p.out = o;
        p.o_bs = (int64_t)Fo * kFrames * Co;
        p.o_xs = (int64_t)Fo * Co;
        p.o_ys = 4LL * Co;
        p.o_off = 0;
        p.a_rounded = conv_rounded(h);  // the DConv output, rounded
        h->gemm(p, PRO_NONE, EPI_STORE, ("dec.convtr" + std::to_string(e)).c_str(), &Dw.convt_all);
      } else {
        // tensor-core builds: all four phases in one GEMM over the input rows
        // (the input read once, not once per phase); output columns
        // phase * Co + c go to row f = 4 f_in + phase of (b, f, t, c)
        ConvParams p = base_params(Dw.convt_all, h->wdev);
        set_input(p, g, G, F, kFrames, C);
        p.B = G;
        p.Hq = F;
        p.Wq = kFrames;
        p.out = o;
        p.o_bs = (int64_t)Fo * kFrames * Co;
        p.o_xs = Co;
        p.o_ys = 4LL * kFrames * Co;
        p.o_off = 0;
        p.o_pcols = Co;
        p.o_pstride = (int64_t)kFrames * Co;
        p.epi_add = skip[j - 1];
        p.a_rounded = conv_rounded(h);  // the DConv output, rounded
        p.round_out = conv_rounded(h);  // feeds only the next decoder's rewrite
        // Only the narrowest of these layers (Cin 96, the largest output) gains: measured on
        // B200, dec.convtr2 1.96 -> 1.19 ms per 42 segments, while at Cin 192 the combined
        // form's zero taps (1.5x the tensor work) made dec.convtr1 slower (0.78 -> 0.96 ms).
        const bool combined =
            C <= 96 &&
            h->gemm_tc(p, EPI_GELU, ("dec.convtr" + std::to_string(e)).c_str(), Dw.convt_all);
        for (int ph = 0; ph < 4 && !combined; ++ph) {
          // (b, f, t, c) with f = 4 f_in + phase
          ConvParams p = base_params(Dw.convt[ph], h->wdev);
          set_input(p, g, G, F, kFrames, C);
          p.B = G;
          p.Hq = F;
          p.Wq = kFrames;
          p.out = o;
          p.o_bs = (int64_t)Fo * kFrames * Co;
          p.o_xs = Co;
          p.o_ys = 4LL * kFrames * Co;
          p.o_off = (int64_t)ph * kFrames * Co;
          p.epi_add = skip[j - 1];
          p.a_rounded = conv_rounded(h);  // the DConv output, rounded
          p.round_out = conv_rounded(h);  // feeds only the next decoder's rewrite
          h->gemm(p, PRO_NONE, EPI_GELU, ("dec.convtr" + std::to_string(e)).c_str(),
                  &Dw.convt[ph]);
        }
      }
      x = o;
      F = Fo;
      C = Co;
      if (last)
        trace_tensor(h, "decoder." + std::to_string(j), x, 3, {G, F, kFrames, C});
      else
        trace_tensor(h, "decoder." + std::to_string(j), x, 0, {G, F, kFrames, C}, skip[j - 1]);
    }
    {  // time decoder (host.rs:763-827)
      const DecW& Dw = m.tdec[e];
      float* g = h->falloc((size_t)G * Tc * Ct);
      ConvParams r = base_params(Dw.rewrite, h->wdev);
      set_input(r, xt, G, 1, Tc, Ct);
      set_output(r, g, G, 1, Tc, Ct);
      r.a_rounded = conv_rounded(h);  // the down-sampler's or previous decoder's output, rounded
      h->gemm(r, PRO_NONE, EPI_GLU, ("tdec.rewrite" + std::to_string(e)).c_str(), &Dw.rewrite);
      run_dconv(h, h->tdec_dc[e], g, G, Tc, conv_rounded(h));
      const int Co = Dw.cout, len = lengths_t[j];
      float* o = h->falloc((size_t)G * len * Co);
      {
        // all four phases in one GEMM over the input positions t: outputs
        // 4t + phase are contiguous in (b, len, c); the last input position's
        // phases beyond len are clipped
        ConvParams p = base_params(Dw.convt_all, h->wdev);
        set_input(p, g, G, 1, Tc, Ct);
        for (int t = 0; t < p.ntaps; ++t) {  // taps move along time for the waveform branch
          p.dx[t] = p.dy[t];
          p.dy[t] = 0;
        }
        p.B = G;
        p.Hq = 1;
        p.Wq = Tc;
        p.out = o;
        p.o_bs = (int64_t)len * Co;
        p.o_xs = 4LL * Co;
        p.o_ys = 0;
        p.o_off = 0;
        p.o_lim = len;
        p.o_lim_ch = Co;
        if (!last) p.epi_add = tskip[j - 1];
        p.a_rounded = conv_rounded(h);               // the DConv output, rounded
        p.round_out = !last && conv_rounded(h);      // feeds only the next decoder's rewrite
        h->gemm(p, PRO_NONE, last ? EPI_STORE : EPI_GELU, ("tdec.convtr" + std::to_string(e)).c_str(),
                &Dw.convt_all);
      }
      xt = o;
      Tc = len;
      Ct = Co;
      trace_tensor(h, "tdecoder." + std::to_string(j), xt, 1, {G, Tc, Ct},
                   last ? nullptr : tskip[j - 1]);
    }
  }

  // (g) iSTFT + branch sum (host.rs:466-519)
  h->mark("spec.istft", 0.0, 4.0 * G * ((double)kBins * kFrames * 16 + 16.0 * L));
  if (h->live()) {
    launch_istft(x, norm_f, h->W(m.window.off), tw, h->W(m.env.off), xt, norm_t, out, G, s);
    h->after("istft");
  }
  h->launches += 1;
}

void check_device_flag(dmx_handle* h) {
  int flag = 0;
  CK(cudaMemcpy(&flag, h->err, sizeof(int), cudaMemcpyDeviceToHost));
  if (flag) {
    CK(cudaMemset(h->err, 0, sizeof(int)));
    throw Error(DMX_ERR_TIMEOUT, std::string(flag == kSelftestCode ? "the self-test kernel"
                                                                   : "a tensor-core kernel") +
                                     " gave up a bounded wait (code " + std::to_string(flag) + ")");
  }
}

void finish_stage_times(dmx_handle* h) {
  if (h->marks.empty()) return;
  CK(cudaEventSynchronize(h->marks.back().ev));
  h->stage_names.clear();
  h->stage_ms.clear();
  h->stage_counts.clear();
  h->stage_flops.clear();
  h->stage_bytes.clear();
  std::map<std::string, size_t> index;
  for (size_t i = 0; i + 1 < h->marks.size(); ++i) {
    const auto& mk = h->marks[i];
    float ms = 0.f;
    CK(cudaEventElapsedTime(&ms, mk.ev, h->marks[i + 1].ev));
    auto it = index.find(mk.name);
    if (it == index.end()) {
      index[mk.name] = h->stage_names.size();
      h->stage_names.push_back(mk.name);
      h->stage_ms.push_back(ms);
      h->stage_counts.push_back(1);
      h->stage_flops.push_back(mk.flops);
      h->stage_bytes.push_back(mk.bytes);
    } else {
      h->stage_ms[it->second] += ms;
      h->stage_counts[it->second] += 1;
      h->stage_flops[it->second] += mk.flops;
      h->stage_bytes[it->second] += mk.bytes;
    }
  }
  for (auto& mk : h->marks) cudaEventDestroy(mk.ev);
  h->marks.clear();
}

void ensure_workspace(dmx_handle* h, int G) {
  const int64_t launches = h->launches;  // the dry run launches nothing
  h->measuring = true;
  h->ws_off = 0;
  h->ws_peak = 0;
  forward(h, nullptr, G, nullptr);
  h->measuring = false;
  h->launches = launches;
  const size_t need = h->ws_peak + (1 << 20);
  if (need > h->ws_cap) {
    if (h->ws) CK(cudaFree(h->ws));
    h->ws = nullptr;
    h->ws_cap = 0;
    CK(cudaMalloc(&h->ws, need));
    h->ws_cap = need;
  }
}

void run_forward(dmx_handle* h, const float* mix_dev, int64_t n, float* out_dev) {
  if (n <= 0) throw Error(DMX_ERR_INVALID, "n_segments must be positive");
  const int cap = std::max(1, h->cfg.max_batch);
  for (int64_t s0 = 0; s0 < n; s0 += cap) {
    const int G = (int)std::min<int64_t>(cap, n - s0);
    ensure_workspace(h, G);
    forward(h, mix_dev + s0 * 2 * kSegment, G, out_dev + s0 * 8 * kSegment);
  }
}

void ensure_io(dmx_handle* h, int64_t n) {
  if (n <= h->io_cap) return;
  cudaFree(h->io_in);
  cudaFree(h->io_out);
  h->io_in = h->io_out = nullptr;
  h->io_cap = 0;
  CK(cudaMalloc(&h->io_in, (size_t)n * 2 * kSegment * sizeof(float)));
  CK(cudaMalloc(&h->io_out, (size_t)n * 8 * kSegment * sizeof(float)));
  h->io_cap = n;
}

}  // namespace dmx
