// Host runtime of the B200 HTDemucs v4 backend: weight ingestion and packing,
// the per-handle workspace, the forward's launch sequence and the C ABI of
// include/dmx.h.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "conv_gemm.cuh"
#include "dmx.h"
#include "tc_gemm.cuh"
#include "kernels.h"

using namespace dmx;

namespace {

thread_local std::string g_error;

struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

#define CK(call)                                                                       \
  do {                                                                                 \
    cudaError_t e_ = (call);                                                           \
    if (e_ != cudaSuccess)                                                             \
      throw Error(e_ == cudaErrorMemoryAllocation ? DMX_ERR_NOMEM : DMX_ERR_CUDA,      \
                  std::string(#call) + ": " + cudaGetErrorString(e_));                 \
  } while (0)

// ---------------------------------------------------------------------------
// safetensors: 8-byte little-endian header size, JSON header, raw data.
// ---------------------------------------------------------------------------
struct HostTensor {
  std::vector<int64_t> shape;
  const float* data = nullptr;                  // into the blob (F32) or into `owned`
  std::shared_ptr<std::vector<float>> owned;  // the f32 copy of a tensor stored in another dtype
  size_t count() const {
    size_t n = 1;
    for (int64_t s : shape) n *= (size_t)s;
    return n;
  }
};

struct Json {
  const char* p;
  const char* end;
  void ws() {
    while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  void expect(char c) {
    ws();
    if (p >= end || *p != c) throw Error(DMX_ERR_WEIGHTS, std::string("safetensors header: expected ") + c);
    ++p;
  }
  bool peek(char c) {
    ws();
    return p < end && *p == c;
  }
  std::string str() {
    expect('"');
    std::string s;
    while (p < end && *p != '"') {
      if (*p == '\\' && p + 1 < end) ++p;
      s += *p++;
    }
    expect('"');
    return s;
  }
  double num() {
    ws();
    char* e = nullptr;
    const double v = strtod(p, &e);
    if (e == p) throw Error(DMX_ERR_WEIGHTS, "safetensors header: expected a number");
    p = e;
    return v;
  }
  void skip() {
    ws();
    if (peek('{')) {
      expect('{');
      if (peek('}')) { expect('}'); return; }
      do { str(); expect(':'); skip(); } while (peek(',') && (expect(','), true));
      expect('}');
    } else if (peek('[')) {
      expect('[');
      if (peek(']')) { expect(']'); return; }
      do { skip(); } while (peek(',') && (expect(','), true));
      expect(']');
    } else if (peek('"')) {
      str();
    } else {
      while (p < end && *p != ',' && *p != '}' && *p != ']') ++p;
    }
  }
};

// IEEE 754 binary16 -> binary32 (subnormals, infinities and NaN included):
// value = (-1)^s * 2^(e-15) * (1 + m/1024), or 2^-14 * m/1024 when e == 0.
float half_bits_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  const uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ff;
  uint32_t bits;
  if (e == 0x1f) {
    bits = sign | 0x7f800000u | (m << 13);  // infinity, or NaN with its payload
  } else if (e != 0) {
    bits = sign | ((e + 112u) << 23) | (m << 13);  // rebias 15 -> 127
  } else {
    float v = (float)m * (1.0f / 16777216.0f);  // m * 2^-24, exact in f32
    std::memcpy(&bits, &v, 4);
    bits |= sign;
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

// Element width of a safetensors dtype this loader reads, 0 if unsupported
// (safetensors.rs:110-135 reads the same set).
int dtype_width(const std::string& d) {
  if (d == "F32" || d == "I32") return 4;
  if (d == "F64" || d == "I64") return 8;
  if (d == "F16" || d == "BF16" || d == "I16") return 2;
  if (d == "U8" || d == "I8" || d == "BOOL") return 1;
  return 0;
}

// Upcasts one non-F32 tensor to f32 (safetensors.rs:110-135).
std::vector<float> decode_tensor(const char* raw, size_t n, const std::string& d) {
  std::vector<float> v(n);
  for (size_t i = 0; i < n; ++i) {
    if (d == "F16" || d == "BF16" || d == "I16") {
      uint16_t u;
      std::memcpy(&u, raw + 2 * i, 2);
      if (d == "F16") {
        v[i] = half_bits_to_float(u);
      } else if (d == "BF16") {
        const uint32_t b = (uint32_t)u << 16;
        std::memcpy(&v[i], &b, 4);
      } else {
        v[i] = (float)(int16_t)u;
      }
    } else if (d == "F64") {
      double x;
      std::memcpy(&x, raw + 8 * i, 8);
      v[i] = (float)x;
    } else if (d == "I64") {
      int64_t x;
      std::memcpy(&x, raw + 8 * i, 8);
      v[i] = (float)x;
    } else if (d == "I32") {
      int32_t x;
      std::memcpy(&x, raw + 4 * i, 4);
      v[i] = (float)x;
    } else if (d == "I8") {
      v[i] = (float)(int8_t)raw[i];
    } else {  // U8, BOOL
      v[i] = (float)(uint8_t)raw[i];
    }
  }
  return v;
}

std::map<std::string, HostTensor> parse_safetensors(const void* blob, size_t len) {
  if (len < 8) throw Error(DMX_ERR_WEIGHTS, "safetensors blob shorter than its header size");
  uint64_t n;
  std::memcpy(&n, blob, 8);
  if (8 + n > len) throw Error(DMX_ERR_WEIGHTS, "safetensors header runs past the blob");
  const char* base = static_cast<const char*>(blob) + 8 + n;
  const size_t data_len = len - 8 - n;
  Json j{static_cast<const char*>(blob) + 8, static_cast<const char*>(blob) + 8 + n};
  std::map<std::string, HostTensor> out;
  j.expect('{');
  if (j.peek('}')) return out;
  while (true) {
    const std::string name = j.str();
    j.expect(':');
    if (name == "__metadata__") {
      j.skip();
    } else {
      HostTensor t;
      std::string dtype;
      size_t a = 0, b = 0;
      j.expect('{');
      while (true) {
        const std::string key = j.str();
        j.expect(':');
        if (key == "dtype") {
          dtype = j.str();
        } else if (key == "shape") {
          j.expect('[');
          if (!j.peek(']')) {
            do { t.shape.push_back((int64_t)j.num()); } while (j.peek(',') && (j.expect(','), true));
          }
          j.expect(']');
        } else if (key == "data_offsets") {
          j.expect('[');
          a = (size_t)j.num();
          j.expect(',');
          b = (size_t)j.num();
          j.expect(']');
        } else {
          j.skip();
        }
        if (j.peek(',')) { j.expect(','); continue; }
        j.expect('}');
        break;
      }
      const int width = dtype_width(dtype);
      if (width == 0) throw Error(DMX_ERR_WEIGHTS, name + ": unsupported safetensors dtype " + dtype);
      if (b < a || b > data_len || b - a != t.count() * (size_t)width)
        throw Error(DMX_ERR_WEIGHTS, name + ": data_offsets do not match the shape");
      if (dtype == "F32" && (reinterpret_cast<uintptr_t>(base + a) & 3) == 0) {
        t.data = reinterpret_cast<const float*>(base + a);
      } else {  // other dtypes (F16 in the published checkpoints), or unaligned F32: an f32 copy
        t.owned = std::make_shared<std::vector<float>>(
            dtype == "F32" ? std::vector<float>(t.count()) : decode_tensor(base + a, t.count(), dtype));
        if (dtype == "F32") std::memcpy(t.owned->data(), base + a, t.count() * 4);
        t.data = t.owned->data();
      }
      out[name] = t;
    }
    if (j.peek(',')) { j.expect(','); continue; }
    j.expect('}');
    break;
  }
  return out;
}

// ---------------------------------------------------------------------------
// Packed weights.
// ---------------------------------------------------------------------------
constexpr int kBK = 16, kBN = 64;

struct Tap {
  int dy, dx;  // input offset of the tap
};

struct Packed {
  size_t w_off = 0, b_off = 0;  // float offsets into the weight arena
  size_t tc_off = 0;            // K-major copy [Npad][K], rounded to nearest tf32
  size_t tc_lo_off = 0;         // its residual w - tf32(w) (3xTF32 split)
  bool has_tc = false;
  int cin = 0;       // input channels as packed (zero rows pad it to a multiple of 16)
  int cin_real = 0;  // the layer's own input channels (for the work count)
  double flop_scale = 1.0;  // algorithmic share of the packed K (structural zeros excluded)
  int K = 0, Kpad = 0, N = 0, Npad = 0;
  std::vector<Tap> taps;
  const float* w = nullptr;
  const float* bias = nullptr;
  // thin first convolutions (K <= 32, 48 outputs): [K][48] then the bias, in
  // host memory, for the kernel that takes them as a launch parameter
  std::vector<float> host_w;
};

struct Vec {  // a plain per-channel vector on the device
  size_t off = 0;
  int n = 0;
  const float* p = nullptr;
};

// fp32 -> nearest tf32 (ties to even), in an fp32 container.
float round_tf32_host(float x) {
  uint32_t b;
  std::memcpy(&b, &x, 4);
  b += 0x0FFFu + ((b >> 13) & 1u);
  b &= 0xFFFFE000u;
  float r;
  std::memcpy(&r, &b, 4);
  return r;
}

struct WeightBuilder {
  std::vector<float> host;
  size_t alloc(size_t n) {
    const size_t off = host.size();
    host.resize(off + ((n + 63) / 64) * 64, 0.f);
    return off;
  }
};

struct EncW {
  Packed conv, rewrite;
  int cin = 0, cout = 0;
};

struct DecW {
  Packed rewrite;
  Packed convt[4];  // per output phase
  Packed convt_all;  // the four phases side by side (see Loader::convt_all)
  int cin = 0, cout = 0;
};

struct LayerW {
  bool cross = false;
  Packed qkv, q, kv, out, lin1, lin2;
  Vec n1w, n1b, n2w, n2b, n3w, n3b, now, nob, g1, g2;
};

struct Model {
  EncW enc[4], tenc[4];
  DecW dec[4], tdec[4];  // execution order
  Packed up, up_t, down, down_t;
  Vec norm_in_w, norm_in_b, norm_in_t_w, norm_in_t_b;
  LayerW layers[5], layers_t[5];
  Vec emb;     // 0.2 * (10 * W)[f, c], (512, 48)
  Vec pos2d;   // (2688, 512)
  Vec pos1d;   // (1344, 512)
  Vec window;  // periodic Hann (4096)
  Vec env;     // window-squared envelope of the interior, (1024)
  Vec ola_w;   // triangular transition weight (segment)
  size_t tw_off = 0;  // float2 twiddles (2048)
};

struct Loader {
  const std::map<std::string, HostTensor>& t;
  WeightBuilder& wb;

  const HostTensor& get(const std::string& name, std::vector<int64_t> shape) {
    auto it = t.find(name);
    if (it == t.end()) throw Error(DMX_ERR_WEIGHTS, "missing tensor " + name);
    if (it->second.shape != shape) {
      std::string s = name + ": shape [";
      for (int64_t d : it->second.shape) s += std::to_string(d) + ",";
      s += "] expected [";
      for (int64_t d : shape) s += std::to_string(d) + ",";
      throw Error(DMX_ERR_WEIGHTS, s + "]");
    }
    return it->second;
  }

  Vec vec(const std::string& name, int n) {
    const HostTensor& h = get(name, {n});
    Vec v;
    v.n = n;
    v.off = wb.alloc(n);
    std::memcpy(&wb.host[v.off], h.data, n * sizeof(float));
    return v;
  }

  // Generic packer: element (tap, ci, column) = value(tap, ci, co(column)).
  template <class F>
  Packed pack(int ntaps, int cin, int cols, bool glu, const float* bias, F value,
              std::vector<Tap> taps) {
    Packed p;
    p.K = ntaps * cin;
    p.Kpad = (p.K + kBK - 1) / kBK * kBK;
    p.N = cols;
    p.Npad = (cols + kBN - 1) / kBN * kBN;
    p.taps = std::move(taps);
    p.cin = cin;
    p.cin_real = cin;
    p.w_off = wb.alloc((size_t)p.Kpad * p.Npad);
    p.b_off = wb.alloc(p.Npad);
    p.has_tc = cin % 16 == 0;
    if (p.has_tc) {
      p.tc_off = wb.alloc((size_t)p.Npad * p.K);
      p.tc_lo_off = wb.alloc((size_t)p.Npad * p.K);
    }
    const int half = cols / 2;
    for (int n = 0; n < cols; ++n) {
      const int co = glu ? ((n % 2 == 0) ? n / 2 : n / 2 + half) : n;
      for (int tap = 0; tap < ntaps; ++tap)
        for (int ci = 0; ci < cin; ++ci) {
          const float v = value(tap, ci, co);
          wb.host[p.w_off + (size_t)(tap * cin + ci) * p.Npad + n] = v;
          if (p.has_tc) {
            const float hi = round_tf32_host(v);
            wb.host[p.tc_off + (size_t)n * p.K + tap * cin + ci] = hi;
            wb.host[p.tc_lo_off + (size_t)n * p.K + tap * cin + ci] = v - hi;
          }
        }
      wb.host[p.b_off + n] = bias[co];
    }
    if (p.K <= 32 && cols == 48 && !glu) {
      p.host_w.resize((size_t)p.K * 48 + 48);
      for (int k = 0; k < p.K; ++k)
        for (int n = 0; n < 48; ++n) p.host_w[(size_t)k * 48 + n] = wb.host[p.w_off + (size_t)k * p.Npad + n];
      for (int n = 0; n < 48; ++n) p.host_w[(size_t)p.K * 48 + n] = wb.host[p.b_off + n];
    }
    return p;
  }

  // Conv (Cout, Cin, kh, kw) with an explicit tap list of (ky, kx) kernel
  // indices and their input offsets.
  Packed conv(const std::string& prefix, std::vector<int64_t> shape,
              const std::vector<std::pair<int, int>>& kidx, std::vector<Tap> taps, bool glu,
              int cin_pad = 0) {
    const HostTensor& w = get(prefix + ".weight", shape);
    const HostTensor& b = get(prefix + ".bias", {shape[0]});
    const int cout = (int)shape[0], cin = (int)shape[1];
    const int kh = shape.size() == 4 ? (int)shape[2] : 1;
    const int kw = shape.size() == 4 ? (int)shape[3] : (int)shape[2];
    Packed p = pack((int)kidx.size(), std::max(cin, cin_pad), cout, glu, b.data,
                    [&](int tap, int ci, int co) {
                      if (ci >= cin) return 0.0f;  // zero rows for padded input channels
                      const int ky = kidx[tap].first, kx = kidx[tap].second;
                      return w.data[(((size_t)co * cin + ci) * kh + ky) * kw + kx];
                    },
                    std::move(taps));
    p.cin_real = cin;
    return p;
  }

  // ConvTranspose (Cin, Cout, k[, 1]) restricted to the two kernel rows that
  // feed output phase `phase` (see the header of convt_taps).
  Packed convt(const std::string& prefix, std::vector<int64_t> shape, int phase) {
    const HostTensor& w = get(prefix + ".weight", shape);
    const int cin = (int)shape[0], cout = (int)shape[1];
    const HostTensor& b = get(prefix + ".bias", {cout});
    const int k = (int)shape[2];
    static const int kf[4][2] = {{2, 6}, {3, 7}, {0, 4}, {1, 5}};
    static const int dq[4][2] = {{0, -1}, {0, -1}, {1, 0}, {1, 0}};
    std::vector<Tap> taps = {{dq[phase][0], 0}, {dq[phase][1], 0}};
    return pack(2, cin, cout, false, b.data,
                [&](int tap, int ci, int co) {
                  return w.data[((size_t)ci * cout + co) * k + kf[phase][tap]];
                },
                taps);
  }

  // All four output phases of the stride-4 ConvTranspose in one GEMM over the
  // input positions q: taps q-1, q, q+1 (K = 3 Cin), columns phase * Cout + co;
  // weights a phase does not use are zero (output 4q + phase reads q + dq).
  Packed convt_all(const std::string& prefix, std::vector<int64_t> shape) {
    const HostTensor& w = get(prefix + ".weight", shape);
    const int cin = (int)shape[0], cout = (int)shape[1];
    const HostTensor& b = get(prefix + ".bias", {cout});
    const int k = (int)shape[2];
    static const int kf[4][2] = {{2, 6}, {3, 7}, {0, 4}, {1, 5}};
    static const int dq[4][2] = {{0, -1}, {0, -1}, {1, 0}, {1, 0}};
    std::vector<float> bias4(4 * (size_t)cout);
    for (int ph = 0; ph < 4; ++ph)
      for (int co = 0; co < cout; ++co) bias4[ph * cout + co] = b.data[co];
    Packed p = pack(3, cin, 4 * cout, false, bias4.data(),
                    [&](int tap, int ci, int n) {
                      const int ph = n / cout, co = n - ph * cout;
                      for (int u = 0; u < 2; ++u)
                        if (dq[ph][u] == tap - 1)
                          return w.data[((size_t)ci * cout + co) * k + kf[ph][u]];
                      return 0.0f;
                    },
                    {{-1, 0}, {0, 0}, {1, 0}});
    p.flop_scale = 2.0 / 3.0;  // each phase uses two of the three taps
    return p;
  }

  Packed linear(const std::string& wname, const std::string& bname, int out, int in, int row0,
                int rows) {
    const HostTensor& w = get(wname, {out, in});
    const HostTensor& b = get(bname, {out});
    return pack(1, in, rows, false, b.data + row0,
                [&](int, int ci, int co) { return w.data[(size_t)(row0 + co) * in + ci]; },
                {{0, 0}});
  }

};

struct DConvLayerW {
  Packed conv1, conv2;
  Vec n1w, n1b, n2w, n2b, gamma;
  std::vector<float> zq;  // the fused tensor-core kernel's moment constants (host memory)
  size_t zq_off = 0;      // the SIMT kernels' moment constants (weight arena)
};

}  // namespace

// ---------------------------------------------------------------------------
// The handle.
// ---------------------------------------------------------------------------
struct DConvFull {
  DConvLayerW layer[2];
  int C = 0, hidden = 0;
};

struct dmx_pending {
  dmx_handle* h;
  int64_t n;
  cudaEvent_t done;
  float* out_dev;
  float* host_pinned;
};

struct dmx_handle {
  dmx_config cfg{};
  int device = 0;
  cudaStream_t stream = nullptr;
  float* wdev = nullptr;
  Model m;
  DConvFull enc_dc[4], tenc_dc[4], dec_dc[4], tdec_dc[4];
  // workspace
  char* ws = nullptr;
  size_t ws_cap = 0, ws_off = 0;
  bool measuring = false;
  size_t ws_peak = 0;
  int64_t launches = 0;
  // io staging
  float* io_in = nullptr;
  float* io_out = nullptr;
  int64_t io_cap = 0;
  float* pinned_in = nullptr;
  float* pinned_out = nullptr;
  dmx_trace_fn trace = nullptr;
  void* trace_user = nullptr;
  bool stage_timing = false;
  struct Mark {
    std::string name;
    cudaEvent_t ev;
    double flops, bytes;  // algorithmic work of the launch that starts here
  };
  std::vector<Mark> marks;
  std::vector<std::string> stage_names;
  std::vector<float> stage_ms;
  std::vector<int> stage_counts;
  std::vector<double> stage_flops, stage_bytes;
  dmx_pending pending{};
  char* track_ws = nullptr;
  size_t track_cap = 0;
  float* host_io = nullptr;  // device staging of dmx_separate_track's host arrays
  size_t host_io_cap = 0;
  double* norm_scratch = nullptr;  // per-block moment partials of dmx_normalize_track_device
  size_t norm_cap = 0;
  int* err = nullptr;  // device flag raised by bounded waits in the tensor-core kernels
  int64_t tc_launches = 0;
  float* bag_out = nullptr;  // this network's own forward output when it runs inside a bag
  int64_t bag_cap = 0;       // segments bag_out holds
  cudaStream_t copy_stream = nullptr;  // device-to-host copies that overlap the forwards
  cudaEvent_t copy_ev = nullptr;
  float* emit_pin[2] = {nullptr, nullptr};  // pinned staging of dmx_separate_track_emit's blocks
  cudaEvent_t emit_ev[2] = {nullptr, nullptr};
  int64_t emit_cap = 0;                     // samples per staging block
  char* batch_ws = nullptr;  // per-track slots of dmx_separate_batch_device
  size_t batch_cap = 0;
  float* tail_buf = nullptr;  // the left neighbour's overlap tail (dmx_separate_track_multi)
  size_t tail_cap = 0;
  cudaEvent_t shard_done = nullptr;  // this handle's chunks are accumulated (multi driver)
  float* batch_io = nullptr;  // device staging of dmx_separate_batch's host tracks and stems
  size_t batch_io_cap = 0;

  float* W(size_t off) const { return wdev + off; }

  void* alloc(size_t bytes) {
    bytes = (bytes + 255) / 256 * 256;
    if (measuring) {
      ws_off += bytes;
      ws_peak = std::max(ws_peak, ws_off);
      return reinterpret_cast<void*>(0x100);
    }
    if (ws_off + bytes > ws_cap) throw Error(DMX_ERR_NOMEM, "workspace exhausted");
    void* p = ws + ws_off;
    ws_off += bytes;
    return p;
  }
  float* falloc(size_t n) { return static_cast<float*>(alloc(n * sizeof(float))); }
  double* dalloc(size_t n) { return static_cast<double*>(alloc(n * sizeof(double))); }

  bool live() const { return !measuring; }

  // Stage timing: an event before each launch, tagged with the launch's
  // algorithmic FLOPs (2 per MAC) and its minimum HBM bytes (each operand read
  // once, each result written once).
  void mark(const std::string& name, double flops = 0.0, double bytes = 0.0) {
    if (!stage_timing || measuring) return;
    cudaEvent_t e;
    CK(cudaEventCreate(&e));
    CK(cudaEventRecord(e, stream));
    marks.push_back({name, e, flops, bytes});
  }

  void zero(void* p, size_t bytes) {
    if (!live()) return;
    CK(cudaMemsetAsync(p, 0, bytes, stream));
  }

  void gemm(const ConvParams& p, int pro, int epi, const char* tag = "gemm",
            const Packed* pk = nullptr) {
    ++launches;
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
    if (pk && (cfg.precision == DMX_TF32 || cfg.precision == DMX_TF32X3) &&
        try_tc(p, pro, epi, *pk))
      return;
    if (pk && !pk->host_w.empty() && launch_first_conv(p, pro, epi, pk->host_w.data(), stream))
      return;
    launch_conv_gemm(p, pro, epi, stream);
  }

  // The tensor-core path alone, for launches the SIMT kernel cannot express
  // (split output columns): false, with nothing launched, when the
  // tensor-core kernel does not take it; the caller then issues another form.
  bool gemm_tc(const ConvParams& p, int epi, const char* tag, const Packed& pk) {
    if (cfg.precision != DMX_TF32 && cfg.precision != DMX_TF32X3) return false;
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
  bool try_tc(const ConvParams& p, int pro, int epi, const Packed& pk) {
    if (pro != PRO_NONE || !pk.has_tc || p.i_cs != 1) return false;
    if (epi != EPI_STORE && epi != EPI_GELU && epi != EPI_GLU && epi != EPI_GLU_EMB &&
        epi != EPI_RESIDUAL)
      return false;
    TcOperandA a;
    TcParams t;
    if (!build_tc(p, pk, a, t)) return false;
    launch_tc_gemm(a, wdev + pk.tc_off,
                   cfg.precision == DMX_TF32X3 ? wdev + pk.tc_lo_off : nullptr, t, epi, stream);
    ++tc_launches;
    return true;
  }

  // ConvParams -> tensor-core operand and parameters; false when unsupported.
  bool build_tc(const ConvParams& p, const Packed& pk, TcOperandA& a, TcParams& t) {
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
    t.epi_gamma = p.epi_gamma;
    t.epi_res = p.epi_res;
    t.epi_emb = p.epi_emb;
    t.epi_add = p.epi_add;
    t.round_out = p.round_out;
    t.vt_out = p.vt_out;
    t.vt_col0 = p.vt_col0;
    t.vt_ntok = p.vt_ntok;
    t.o_lim = p.o_lim;
    t.o_lim_ch = p.o_lim_ch;
    t.a_rounded = p.a_rounded;
    t.o_pcols = p.o_pcols;
    t.o_pstride = p.o_pstride;
    t.err = err;
    return tc_gemm_supported(a, t);
  }

  void after(const char* what) {
    if (!live()) return;
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) throw Error(DMX_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  }
};

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
  launch_tc_gemm(a, h->W(pk.tc_off), h->W(pk.tc_lo_off), t, epi, h->stream);
  ++h->tc_launches;
}

// The DConv branch as two persistent tensor-core GEMMs per layer around a
// SIMT pass, for rows of any length: conv1 (taps as TMA offsets) storing y
// and its row moments; the row moments of z from g = GELU(GroupNorm1(y)) by
// the quadratic form (dconv.cu); conv2 with GELU(GroupNorm1(y)) applied to
// each A tile by the converter warps and a GroupNorm2 + GLU + LayerScale +
// residual epilogue into x. Moments are f64 atomics per row.
void run_dconv_gemm(dmx_handle* h, const DConvFull& dc, float* x, int rows, int T,
                    bool round_out) {
  const int C = dc.C, hid = dc.hidden;
  const int64_t positions = (int64_t)rows * T;
  const int kg = dc.layer[0].conv2.K;  // y row width = conv2's padded K
  float* y = h->falloc((size_t)positions * kg);
  double* st = h->dalloc((size_t)rows * 4);
  for (int d = 0; d < 2; ++d) {
    const DConvLayerW& L = dc.layer[d];
    h->mark("dconv.gemm" + std::to_string(C), 10.0 * positions * C * hid, 8.0 * positions * C);
    h->launches += 3;
    if (!h->live()) continue;
    CK(cudaMemsetAsync(st, 0, (size_t)rows * 4 * sizeof(double), h->stream));
    TcParams ext;
    std::memset(&ext, 0, sizeof(ext));
    {  // conv1: x (rows, T, C) -> y (rows, T, kg), the first hid columns
      ConvParams p = base_params(L.conv1, h->wdev);
      set_input(p, x, rows, 1, T, C);
      set_output(p, y, rows, 1, T, kg);
      p.epi_stats = st;
      p.epi_rowlen = T;
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
                             h->W(L.zq_off), h->stream))
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

// round_out: the branch's output feeds only a tf32 GEMM (the TF32 build): the
// last layer stores it rounded to nearest tf32 so that GEMM needs no converter.
void run_dconv(dmx_handle* h, const DConvFull& dc, float* x, int rows, int T, bool round_out) {
  const int C = dc.C, hid = dc.hidden;
  const int64_t positions = (int64_t)rows * T;
  const bool tf32 = h->cfg.precision == DMX_TF32 || h->cfg.precision == DMX_TF32X3;
  const bool has_tc = dc.layer[0].conv1.has_tc && dc.layer[0].conv2.has_tc;
  // TF32 builds: tensor cores (3xTF32, fp32-accurate) for the narrow layers
  // (the fused kernel: one launch per spectral row, three over the tiles of a
  // waveform row) and the widest layers (three GEMMs, where the SIMT kernels
  // are compute-bound); the SIMT kernels are faster elsewhere
  const bool tc = tf32 && has_tc && !dc.layer[0].zq.empty() && dconv_tc_supported(C, T);
  if (tf32 && has_tc && !tc && C >= 384) {
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

void xf_gemm(dmx_handle* h, const char* tag, const Packed& pk, const float* in, int B, int n,
             float* out, int epi, const float* res = nullptr, const float* gamma = nullptr,
             double* stats = nullptr, bool round_out = false, float* vt = nullptr,
             int vt_col0 = 0) {
  ConvParams p = base_params(pk, h->wdev);
  p.round_out = round_out;
  p.a_rounded = xf_rounded(h);
  p.vt_out = vt;
  p.vt_col0 = vt_col0;
  p.vt_ntok = n;
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
                      xf_rounded(h));
  ++h->launches;
  xf_gemm(h, "xf.ffn1", L.lin1, bb.xn, B, n, bb.hid, EPI_GELU, nullptr, nullptr, nullptr,
          xf_rounded(h));
  h->zero(bb.stats, (size_t)B * 2 * sizeof(double));
  xf_gemm(h, "xf.ffn2", L.lin2, bb.hid, B, n, X, EPI_RESIDUAL, X, h->W(L.g2.off), bb.stats);
  h->mark("xf.groupnorm", 0.0, 8.0 * B * n * 512);
  if (h->live()) launch_group_norm_apply(X, B, n, bb.stats, h->W(L.now.off), h->W(L.nob.off), h->stream);
  ++h->launches;
}

void xf_self(dmx_handle* h, const LayerW& L, float* X, int B, int n, const XfBufs& bb) {
  h->mark("xf.layernorm", 0.0, 8.0 * B * n * 512);
  if (h->live()) launch_layer_norm(X, (int64_t)B * n, n, h->W(L.n1w.off), h->W(L.n1b.off), nullptr, bb.xn,
                                   h->stream, xf_rounded(h));
  ++h->launches;
  const bool tc_attn = h->cfg.precision == DMX_TF32;
  xf_gemm(h, "xf.qkv", L.qkv, bb.xn, B, n, bb.qkv, EPI_STORE, nullptr, nullptr, nullptr, tc_attn,
          tc_attn ? bb.vt1 : nullptr, 1024);
  h->mark("xf.attention", 4.0 * B * n * n * 512, 4.0 * B * n * 512 * 4);
  if (h->live() && !(tc_attn && launch_attention_tc(bb.qkv, 1536, 0, bb.qkv, 1536, 512, 1024, bb.vt1,
                                                     bb.att, 512, B, 8, n, n, 0.125f, h->err,
                                                     h->stream)))
    launch_flash_attention(bb.qkv, 1536, bb.qkv + 512, bb.qkv + 1024, 1536, bb.att, 512, B, 8, n, n,
                           0.125f, h->stream);
  ++h->launches;
  xf_tail(h, L, X, B, n, bb, L.n2w, L.n2b);
}

// kv projection of the other stream for a cross layer (LN2 of this layer).
void xf_cross_kv(dmx_handle* h, const LayerW& L, const float* other, int B, int n_other,
                 float* kv_out, float* scratch, float* vt) {
  h->mark("xf.layernorm", 0.0, 8.0 * B * n_other * 512);
  if (h->live())
    launch_layer_norm(other, (int64_t)B * n_other, n_other, h->W(L.n2w.off), h->W(L.n2b.off), nullptr,
                      scratch, h->stream, xf_rounded(h));
  ++h->launches;
  const bool tc_attn = h->cfg.precision == DMX_TF32;
  xf_gemm(h, "xf.kv", L.kv, scratch, B, n_other, kv_out, EPI_STORE, nullptr, nullptr, nullptr,
          tc_attn, tc_attn ? vt : nullptr, 512);
}

void xf_cross(dmx_handle* h, const LayerW& L, float* X, int B, int n, const float* kv,
              const float* vt, int n_other, const XfBufs& bb) {
  h->mark("xf.layernorm", 0.0, 8.0 * B * n * 512);
  if (h->live()) launch_layer_norm(X, (int64_t)B * n, n, h->W(L.n1w.off), h->W(L.n1b.off), nullptr, bb.xn,
                                   h->stream, xf_rounded(h));
  ++h->launches;
  const bool tc_attn = h->cfg.precision == DMX_TF32;
  xf_gemm(h, "xf.q", L.q, bb.xn, B, n, bb.qkv, EPI_STORE, nullptr, nullptr, nullptr, tc_attn);
  h->mark("xf.attention", 4.0 * B * n * n_other * 512, 4.0 * B * (2.0 * n + 2.0 * n_other) * 512);
  if (h->live() && !(tc_attn && launch_attention_tc(bb.qkv, 512, 0, kv, 1024, 0, 512, vt, bb.att,
                                                     512, B, 8, n, n_other, 0.125f, h->err,
                                                     h->stream)))
    launch_flash_attention(bb.qkv, 512, kv, kv + 512, 1024, bb.att, 512, B, 8, n, n_other, 0.125f,
                           h->stream);
  ++h->launches;
  xf_tail(h, L, X, B, n, bb, L.n3w, L.n3b);
}

// The whole forward of G segments: mix (G, 2, L) device, normalised chunks ->
// out (G, 4, 2, L) device (Htdemucs::forward, host.rs:202-520).
void forward(dmx_handle* h, const float* mix, int G, float* out) {
  const int L = kSegment;
  const Model& m = h->m;
  h->ws_off = 0;
  cudaStream_t s = h->stream;
  const float2* tw = reinterpret_cast<const float2*>(h->W(m.tw_off));

  // (a) spectrogram + moments
  double* mom = h->dalloc((size_t)G * 4);
  float4* norm = static_cast<float4*>(h->alloc((size_t)G * 2 * sizeof(float4)));
  float4* norm_f = norm;
  float4* norm_t = norm + G;
  float* X = h->falloc((size_t)G * kBins * kFrames * 4);
  h->zero(mom, (size_t)G * 4 * sizeof(double));
  h->mark("spec.stft", 0.0, 4.0 * G * (2.0 * L + (double)kBins * kFrames * 4));
  if (h->live()) {
    launch_stft_cac(mix, G, h->W(m.window.off), tw, X, mom, s);
    launch_wave_moments(mix, G, 2LL * L, mom + 2 * G, s);
    launch_norm_finalize(mom, (double)kBins * kFrames * 4, G, norm_f, s);
    launch_norm_finalize(mom + 2 * G, 2.0 * L, G, norm_t, s);
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
      run_dconv(h, h->tenc_dc[i], y, G, To, xf_rounded(h));
      float* z = h->falloc((size_t)G * To * Co);
      ConvParams r = base_params(E.rewrite, h->wdev);
      set_input(r, y, G, 1, To, Co);
      set_output(r, z, G, 1, To, Co);
      r.a_rounded = xf_rounded(h);  // the DConv output, rounded
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
      run_dconv(h, h->enc_dc[i], y, G * Fo, kFrames, xf_rounded(h));
      float* z = h->falloc((size_t)G * Fo * kFrames * Co);
      ConvParams r = base_params(E.rewrite, h->wdev);
      set_input(r, y, G, Fo, kFrames, Co);
      set_output(r, z, G, Fo, kFrames, Co);
      if (i == 0) r.epi_emb = h->W(m.emb.off);
      r.a_rounded = xf_rounded(h);  // the DConv output, rounded
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
    p.round_out = xf_rounded(h);  // feeds only the first decoder's rewrite
    h->gemm(p, PRO_NONE, EPI_STORE, "xf.downsample", &m.down);
    ConvParams q = base_params(m.down_t, h->wdev);
    set_input(q, Tk, G, 1, Tt, D);
    set_output(q, xt, G, 1, Tt, TCs[4]);
    q.epi_add = tskip[3];
    q.round_out = xf_rounded(h);
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
      r.a_rounded = xf_rounded(h);  // the down-sampler's or previous decoder's output, rounded
      h->gemm(r, PRO_NONE, EPI_GLU, ("dec.rewrite" + std::to_string(e)).c_str(), &Dw.rewrite);
      run_dconv(h, h->dec_dc[e], g, G * F, kFrames, xf_rounded(h));
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
        p.a_rounded = xf_rounded(h);  // the DConv output, rounded
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
        p.a_rounded = xf_rounded(h);  // the DConv output, rounded
        p.round_out = xf_rounded(h);  // feeds only the next decoder's rewrite
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
          p.a_rounded = xf_rounded(h);  // the DConv output, rounded
          p.round_out = xf_rounded(h);  // feeds only the next decoder's rewrite
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
      r.a_rounded = xf_rounded(h);  // the down-sampler's or previous decoder's output, rounded
      h->gemm(r, PRO_NONE, EPI_GLU, ("tdec.rewrite" + std::to_string(e)).c_str(), &Dw.rewrite);
      run_dconv(h, h->tdec_dc[e], g, G, Tc, xf_rounded(h));
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
        p.a_rounded = xf_rounded(h);               // the DConv output, rounded
        p.round_out = !last && xf_rounded(h);      // feeds only the next decoder's rewrite
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

// Raises DMX_ERR_TIMEOUT when a tensor-core kernel gave up a bounded wait.
constexpr int kSelftestCode = 99;  // the error code dmx_selftest_wait_timeout's kernel raises

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

// Sizes the workspace for `G` segments by a dry run of the launch sequence.
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

void load_model(dmx_handle* h, const std::map<std::string, HostTensor>& t) {
  WeightBuilder wb;
  Loader L{t, wb};
  Model& m = h->m;
  auto line8 = [](bool along_h) {
    std::vector<std::pair<int, int>> k;
    std::vector<Tap> taps;
    for (int i = 0; i < 8; ++i) {
      k.emplace_back(along_h ? i : 0, along_h ? 0 : i);
      taps.push_back(along_h ? Tap{i - 2, 0} : Tap{0, i - 2});
    }
    return std::make_pair(k, taps);
  };
  // The fused tensor-core DConv kernel (C = 48, 96) reads its hidden channels
  // in K slots (dconv_tc_slot): conv1's output rows and conv2's input columns
  // of the tensor-core copies move there, and the moments of conv2's output
  // get their host-side constants v = sum_c w_c, M = sum_c w_c w_c'.
  auto tc_dconv_slots = [&](int C, DConvLayerW& Lw) {
    const int hid = C / 8, act = hid + 1;
    int src[16];  // slot -> old slot (hidden channel h sat at h, the bias at 15)
    for (int k = 0; k < 16; ++k) src[k] = -1;
    for (int i = 0; i < act; ++i) src[dconv_tc_slot(hid, i)] = i < hid ? i : 15;
    const Packed& p1 = Lw.conv1;
    for (size_t off : {p1.tc_off, p1.tc_lo_off}) {
      std::vector<float> old(wb.host.begin() + off, wb.host.begin() + off + (size_t)16 * p1.K);
      for (int k = 0; k < 16; ++k)
        for (int j = 0; j < p1.K; ++j)
          wb.host[off + (size_t)k * p1.K + j] = src[k] >= 0 && src[k] < hid ? old[(size_t)src[k] * p1.K + j] : 0.f;
    }
    const Packed& p2 = Lw.conv2;
    for (size_t off : {p2.tc_off, p2.tc_lo_off})
      for (int n = 0; n < 2 * C; ++n) {
        float* row = &wb.host[off + (size_t)n * 16];
        float old[16];
        std::copy(row, row + 16, old);
        for (int k = 0; k < 16; ++k) row[k] = src[k] >= 0 ? old[src[k]] : 0.f;
      }
    std::vector<double> w((size_t)2 * C * act);
    for (int n = 0; n < 2 * C; ++n)
      for (int i = 0; i < act; ++i) {
        const size_t e = (size_t)n * 16 + dconv_tc_slot(hid, i);
        w[(size_t)n * act + i] = (double)wb.host[p2.tc_off + e] + (double)wb.host[p2.tc_lo_off + e];
      }
    Lw.zq.assign(dconv_tc_const_floats(C), 0.f);
    for (int i = 0; i < act; ++i) {
      double v = 0.0;
      for (int n = 0; n < 2 * C; ++n) v += w[(size_t)n * act + i];
      Lw.zq[i] = (float)v;
    }
    for (int i = 0, idx = act; i < act; ++i)
      for (int j = i; j < act; ++j, ++idx) {
        double m = 0.0;
        for (int n = 0; n < 2 * C; ++n) m += w[(size_t)n * act + i] * w[(size_t)n * act + j];
        Lw.zq[idx] = (float)(i == j ? m : 2.0 * m);
      }
    float* tail = Lw.zq.data() + act + act * (act + 1) / 2;
    for (int h = 0; h < hid; ++h) {
      tail[h] = wb.host[Lw.conv1.b_off + h];
      tail[hid + h] = wb.host[Lw.n1w.off + h];
      tail[2 * hid + h] = wb.host[Lw.n1b.off + h];
    }
  };
  // The SIMT DConv kernels' GroupNorm2 moments from g: w~_n = (conv2 column
  // n's weights, its bias) over all 2C columns; v = sum_n w~_n and
  // M = sum_n w~_n w~_n' (f64, stored as f32).
  auto simt_dconv_moments = [&](int C, DConvLayerW& Lw) {
    const int hid = C / 8, act = hid + 1;
    const Packed& p2 = Lw.conv2;
    std::vector<double> w((size_t)2 * C * act);
    for (int n = 0; n < 2 * C; ++n) {
      for (int h = 0; h < hid; ++h) w[(size_t)n * act + h] = wb.host[p2.w_off + (size_t)h * p2.Npad + n];
      w[(size_t)n * act + hid] = wb.host[p2.b_off + n];
    }
    const int ld = dconv_zq_stride(C);
    Lw.zq_off = wb.alloc(dconv_zq_floats(C));
    float* z = &wb.host[Lw.zq_off];  // zero filled by alloc
    for (int i = 0; i < act; ++i) {
      double v = 0.0;
      for (int n = 0; n < 2 * C; ++n) v += w[(size_t)n * act + i];
      z[i] = (float)v;
    }
    for (int i = 0; i < act; ++i)
      for (int j = 0; j < act; ++j) {
        double m = 0.0;
        for (int n = 0; n < 2 * C; ++n) m += w[(size_t)n * act + i] * w[(size_t)n * act + j];
        z[(size_t)ld * (1 + i) + j] = (float)m;
      }
  };
  auto load_dc = [&](const std::string& prefix, int C, DConvFull* dc) {
    dc->C = C;
    dc->hidden = C / 8;
    for (int d = 0; d < 2; ++d) {
      const std::string at = prefix + ".dconv.layers." + std::to_string(d);
      const int dil = 1 << d;
      DConvLayerW& Lw = dc->layer[d];
      Lw.conv1 = L.conv(at + ".0", {C / 8, C, 3}, {{0, 0}, {0, 1}, {0, 2}},
                        {{0, -dil}, {0, 0}, {0, dil}}, false);
      Lw.n1w = L.vec(at + ".1.weight", C / 8);
      Lw.n1b = L.vec(at + ".1.bias", C / 8);
      Lw.conv2 = L.conv(at + ".3", {2 * C, C / 8, 1}, {{0, 0}}, {{0, 0}}, true,
                        (C / 8 + 15) / 16 * 16);
      // tensor-core copy of conv2 (used only by the fused DConv kernel): the
      // bias rides in the last, zero-padded input channel, which that kernel
      // feeds with 1
      if (Lw.conv2.has_tc && C / 8 < Lw.conv2.K) {
        const int kb = Lw.conv2.K - 1;
        for (int n = 0; n < 2 * C; ++n) {
          const float b = wb.host[Lw.conv2.b_off + n];
          const float hi = round_tf32_host(b);
          wb.host[Lw.conv2.tc_off + (size_t)n * Lw.conv2.K + kb] = hi;
          wb.host[Lw.conv2.tc_lo_off + (size_t)n * Lw.conv2.K + kb] = b - hi;
        }
      }
      if ((C == 48 || C == 96) && Lw.conv1.has_tc && Lw.conv2.has_tc && Lw.conv2.K == 16)
        tc_dconv_slots(C, Lw);
      simt_dconv_moments(C, Lw);
      Lw.n2w = L.vec(at + ".4.weight", 2 * C);
      Lw.n2b = L.vec(at + ".4.bias", 2 * C);
      Lw.gamma = L.vec(at + ".6.scale", C);
    }
  };
  int chin_z = 4, chin = 2, chout = 48;
  for (int i = 0; i < 4; ++i) {
    const std::string e = "encoder." + std::to_string(i), te = "tencoder." + std::to_string(i);
    auto fl = line8(true);
    m.enc[i].conv = L.conv(e + ".conv", {chout, chin_z, 8, 1}, fl.first, fl.second, false);
    m.enc[i].rewrite = L.conv(e + ".rewrite", {2 * chout, chout, 1, 1}, {{0, 0}}, {{0, 0}}, true);
    m.enc[i].cin = chin_z;
    m.enc[i].cout = chout;
    load_dc(e, chout, &h->enc_dc[i]);
    auto tl = line8(false);
    m.tenc[i].conv = L.conv(te + ".conv", {chout, chin, 8}, tl.first, tl.second, false);
    m.tenc[i].rewrite = L.conv(te + ".rewrite", {2 * chout, chout, 1}, {{0, 0}}, {{0, 0}}, true);
    m.tenc[i].cin = chin;
    m.tenc[i].cout = chout;
    load_dc(te, chout, &h->tenc_dc[i]);
    chin_z = chin = chout;
    chout *= 2;
  }
  for (int e = 0; e < 4; ++e) {
    const int j = 3 - e;
    const int cin = 48 << j;
    const int cout_f = j == 0 ? 16 : 48 << (j - 1);
    const int cout_t = j == 0 ? 8 : 48 << (j - 1);
    const std::string d = "decoder." + std::to_string(j), td = "tdecoder." + std::to_string(j);
    std::vector<std::pair<int, int>> k9;
    std::vector<Tap> t9;
    for (int ky = 0; ky < 3; ++ky)
      for (int kx = 0; kx < 3; ++kx) {
        k9.emplace_back(ky, kx);
        t9.push_back({ky - 1, kx - 1});
      }
    m.dec[e].rewrite = L.conv(d + ".rewrite", {2 * cin, cin, 3, 3}, k9, t9, true);
    // all four phases in one GEMM: the last decoder writes the frame-major
    // spectrogram (phases contiguous), the others split the columns per phase
    m.dec[e].convt_all = L.convt_all(d + ".conv_tr", {cin, cout_f, 8, 1});
    if (e != 3)  // per-phase GEMMs: the FP32 (SIMT) build
      for (int ph = 0; ph < 4; ++ph)
        m.dec[e].convt[ph] = L.convt(d + ".conv_tr", {cin, cout_f, 8, 1}, ph);
    m.dec[e].cin = cin;
    m.dec[e].cout = cout_f;
    load_dc(d, cin, &h->dec_dc[e]);
    m.tdec[e].rewrite = L.conv(td + ".rewrite", {2 * cin, cin, 3}, {{0, 0}, {0, 1}, {0, 2}},
                               {{0, -1}, {0, 0}, {0, 1}}, true);
    m.tdec[e].convt_all = L.convt_all(td + ".conv_tr", {cin, cout_t, 8});
    m.tdec[e].cin = cin;
    m.tdec[e].cout = cout_t;
    load_dc(td, cin, &h->tdec_dc[e]);
  }
  m.up = L.conv("channel_upsampler", {512, 384, 1}, {{0, 0}}, {{0, 0}}, false);
  m.up_t = L.conv("channel_upsampler_t", {512, 384, 1}, {{0, 0}}, {{0, 0}}, false);
  m.down = L.conv("channel_downsampler", {384, 512, 1}, {{0, 0}}, {{0, 0}}, false);
  m.down_t = L.conv("channel_downsampler_t", {384, 512, 1}, {{0, 0}}, {{0, 0}}, false);
  m.norm_in_w = L.vec("crosstransformer.norm_in.weight", 512);
  m.norm_in_b = L.vec("crosstransformer.norm_in.bias", 512);
  m.norm_in_t_w = L.vec("crosstransformer.norm_in_t.weight", 512);
  m.norm_in_t_b = L.vec("crosstransformer.norm_in_t.bias", 512);
  for (int s = 0; s < 2; ++s)
    for (int l = 0; l < 5; ++l) {
      LayerW& Lw = s == 0 ? m.layers[l] : m.layers_t[l];
      const std::string at = std::string("crosstransformer.") + (s == 0 ? "layers." : "layers_t.") + std::to_string(l);
      Lw.cross = l % 2 == 1;
      const std::string attn = at + (Lw.cross ? ".cross_attn" : ".self_attn");
      if (Lw.cross) {
        Lw.q = L.linear(attn + ".in_proj_weight", attn + ".in_proj_bias", 1536, 512, 0, 512);
        Lw.kv = L.linear(attn + ".in_proj_weight", attn + ".in_proj_bias", 1536, 512, 512, 1024);
        Lw.n3w = L.vec(at + ".norm3.weight", 512);
        Lw.n3b = L.vec(at + ".norm3.bias", 512);
      } else {
        Lw.qkv = L.linear(attn + ".in_proj_weight", attn + ".in_proj_bias", 1536, 512, 0, 1536);
      }
      Lw.out = L.linear(attn + ".out_proj.weight", attn + ".out_proj.bias", 512, 512, 0, 512);
      Lw.lin1 = L.linear(at + ".linear1.weight", at + ".linear1.bias", 2048, 512, 0, 2048);
      Lw.lin2 = L.linear(at + ".linear2.weight", at + ".linear2.bias", 512, 2048, 0, 512);
      Lw.n1w = L.vec(at + ".norm1.weight", 512);
      Lw.n1b = L.vec(at + ".norm1.bias", 512);
      Lw.n2w = L.vec(at + ".norm2.weight", 512);
      Lw.n2b = L.vec(at + ".norm2.bias", 512);
      Lw.now = L.vec(at + ".norm_out.weight", 512);
      Lw.nob = L.vec(at + ".norm_out.bias", 512);
      Lw.g1 = L.vec(at + ".gamma_1.scale", 512);
      Lw.g2 = L.vec(at + ".gamma_2.scale", 512);
    }
  // Tables computed on the host in f32 exactly as the reference does.
  {
    const HostTensor& e = L.get("freq_emb.embedding.weight", {512, 48});
    m.emb.n = 512 * 48;
    m.emb.off = wb.alloc(m.emb.n);
    for (int i = 0; i < m.emb.n; ++i) wb.host[m.emb.off + i] = 0.2f * (e.data[i] * 10.0f);
  }
  {  // create_2d_sin_embedding (host.rs:1078-1106): token t*8 + f
    const int dim = 512, half = 256, pairs = 128, height = 8, width = 336;
    const float log_period = std::log(10000.0f) / (float)half;
    std::vector<float> div(pairs);
    for (int jj = 0; jj < pairs; ++jj) div[jj] = std::exp(-((float)(2 * jj)) * log_period);
    m.pos2d.n = width * height * dim;
    m.pos2d.off = wb.alloc(m.pos2d.n);
    for (int t = 0; t < width; ++t)
      for (int f = 0; f < height; ++f) {
        float* o = &wb.host[m.pos2d.off + ((size_t)t * height + f) * dim];
        for (int jj = 0; jj < pairs; ++jj) {
          const float w = (float)t * div[jj], hh = (float)f * div[jj];
          o[2 * jj] = std::sin(w);
          o[2 * jj + 1] = std::cos(w);
          o[half + 2 * jj] = std::sin(hh);
          o[half + 2 * jj + 1] = std::cos(hh);
        }
      }
  }
  {  // create_sin_embedding (host.rs:1110-1122)
    const int length = 1344, dim = 512, half = 256;
    m.pos1d.n = length * dim;
    m.pos1d.off = wb.alloc(m.pos1d.n);
    for (int t = 0; t < length; ++t)
      for (int i = 0; i < half; ++i) {
        const float exponent = (float)i / ((float)half - 1.0f);
        const float phase = (float)t / std::pow(10000.0f, exponent);
        wb.host[m.pos1d.off + (size_t)t * dim + i] = std::cos(phase);
        wb.host[m.pos1d.off + (size_t)t * dim + half + i] = std::sin(phase);
      }
  }
  {  // periodic Hann (stft.rs:54-61), envelope, twiddles, OLA weight
    m.window.n = kNfft;
    m.window.off = wb.alloc(kNfft);
    for (int i = 0; i < kNfft; ++i)
      wb.host[m.window.off + i] = (float)(0.5 - 0.5 * std::cos(2.0 * M_PI * (double)i / (double)kNfft));
    m.env.n = kHop;
    m.env.off = wb.alloc(kHop);
    for (int r = 0; r < kHop; ++r) {
      float env = 0.f;  // frames in increasing order: offsets r+3072 .. r
      for (int k = 3; k >= 0; --k) {
        const float w = wb.host[m.window.off + r + k * kHop];
        env += w * w;
      }
      wb.host[m.env.off + r] = env;
    }
    m.tw_off = wb.alloc(2 * 2048);
    for (int k = 0; k < 2048; ++k) {
      const double a = 2.0 * M_PI * (double)k / (double)kNfft;
      wb.host[m.tw_off + 2 * k] = (float)std::cos(a);
      wb.host[m.tw_off + 2 * k + 1] = (float)-std::sin(a);
    }
    // transition_weight(segment, 1.0) (pipeline.rs:117-131)
    const int seg = h->cfg.segment_samples, half = seg / 2;
    m.ola_w.n = seg;
    m.ola_w.off = wb.alloc(seg);
    for (int i = 0; i < seg; ++i)
      wb.host[m.ola_w.off + i] = (float)(i < half ? i + 1 : seg - i);
    const float mx = std::max((float)std::max(half, seg - half), 1.0f);
    for (int i = 0; i < seg; ++i) wb.host[m.ola_w.off + i] = wb.host[m.ola_w.off + i] / mx;
  }
  CK(cudaMalloc(&h->wdev, wb.host.size() * sizeof(float)));
  CK(cudaMemcpy(h->wdev, wb.host.data(), wb.host.size() * sizeof(float), cudaMemcpyHostToDevice));
}

int fail(const Error& e) {
  g_error = e.what();
  return e.code;
}
int fail_std(const std::exception& e) {
  g_error = e.what();
  return DMX_ERR_INVALID;
}

}  // namespace

// Lets other translation units (noalloc.cu) report through dmx_last_error.
void dmx::set_last_error(const char* msg) { g_error = msg; }

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
extern "C" {

void dmx_default_config(dmx_config* c) {
  c->sources = 4;
  c->audio_channels = 2;
  c->samplerate = 44100;
  c->segment_samples = kSegment;
  c->precision = DMX_FP32;
  c->max_batch = 8;
}

const char* dmx_last_error(void) { return g_error.c_str(); }

dmx_status dmx_create(const dmx_config* cfg, const void* blob, size_t len, int device,
                      dmx_handle** out) {
  if (!cfg || !blob || !out) {
    g_error = "dmx_create: null argument";
    return DMX_ERR_INVALID;
  }
  std::unique_ptr<dmx_handle> h(new dmx_handle());
  try {
    if (cfg->sources != 4 || cfg->audio_channels != 2 || cfg->samplerate != 44100 ||
        cfg->segment_samples != kSegment)
      throw Error(DMX_ERR_INVALID,
                  "only the default htdemucs configuration is supported (4 sources, stereo, "
                  "44100 Hz, 343980-sample segments)");
    if (cfg->precision != DMX_FP32 && cfg->precision != DMX_TF32 &&
        cfg->precision != DMX_TF32X3)
      throw Error(DMX_ERR_INVALID, "precision must be DMX_FP32, DMX_TF32 or DMX_TF32X3");
    if (cfg->max_batch < 1 || cfg->max_batch > 256)
      throw Error(DMX_ERR_INVALID, "max_batch must be in [1, 256]");
    h->cfg = *cfg;
    h->device = device;
    const auto tensors = parse_safetensors(blob, len);  // validated before any CUDA call
    CK(cudaSetDevice(device));
    CK(cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking));
    CK(cudaMalloc(&h->err, sizeof(int)));
    CK(cudaMemset(h->err, 0, sizeof(int)));
    load_model(h.get(), tensors);
    const char* st = getenv("DMX_STAGE_TIMING");
    h->stage_timing = st && st[0] == '1';
    *out = h.release();
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

void dmx_destroy(dmx_handle* h) {
  if (!h) return;
  cudaSetDevice(h->device);
  if (h->stream) cudaStreamSynchronize(h->stream);
  if (h->pending.done) cudaEventDestroy(h->pending.done);
  cudaFree(h->wdev);
  cudaFree(h->err);
  cudaFree(h->ws);
  cudaFree(h->io_in);
  cudaFree(h->io_out);
  cudaFree(h->track_ws);
  cudaFree(h->host_io);
  cudaFree(h->norm_scratch);
  cudaFree(h->bag_out);
  if (h->copy_stream) cudaStreamSynchronize(h->copy_stream);
  if (h->copy_ev) cudaEventDestroy(h->copy_ev);
  for (int i = 0; i < 2; ++i) {
    if (h->emit_ev[i]) cudaEventDestroy(h->emit_ev[i]);
    cudaFreeHost(h->emit_pin[i]);
  }
  if (h->copy_stream) cudaStreamDestroy(h->copy_stream);
  cudaFree(h->batch_ws);
  cudaFree(h->tail_buf);
  if (h->shard_done) cudaEventDestroy(h->shard_done);
  cudaFree(h->batch_io);
  cudaFreeHost(h->pinned_in);
  cudaFreeHost(h->pinned_out);
  if (h->stream) cudaStreamDestroy(h->stream);
  delete h;
}

dmx_status dmx_set_trace(dmx_handle* h, dmx_trace_fn fn, void* user) {
  if (!h) return DMX_ERR_INVALID;
  h->trace = fn;
  h->trace_user = user;
  return DMX_OK;
}

dmx_status dmx_forward_device(dmx_handle* h, const float* mix_dev, int64_t n, float* out_dev,
                              void* stream) {
  try {
    CK(cudaSetDevice(h->device));
    h->launches = 0;
    cudaStream_t user = static_cast<cudaStream_t>(stream);
    if (user && user != h->stream) {
      cudaEvent_t e;
      CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
      CK(cudaEventRecord(e, user));
      CK(cudaStreamWaitEvent(h->stream, e, 0));
      run_forward(h, mix_dev, n, out_dev);
      CK(cudaEventRecord(e, h->stream));
      CK(cudaStreamWaitEvent(user, e, 0));
      CK(cudaEventDestroy(e));
    } else {
      run_forward(h, mix_dev, n, out_dev);
    }
    h->mark("end");
    finish_stage_times(h);
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

static void ensure_io(dmx_handle* h, int64_t n) {
  if (n <= h->io_cap) return;
  cudaFree(h->io_in);
  cudaFree(h->io_out);
  cudaFreeHost(h->pinned_in);
  cudaFreeHost(h->pinned_out);
  h->io_in = h->io_out = h->pinned_in = h->pinned_out = nullptr;
  CK(cudaMalloc(&h->io_in, (size_t)n * 2 * kSegment * sizeof(float)));
  CK(cudaMalloc(&h->io_out, (size_t)n * 8 * kSegment * sizeof(float)));
  CK(cudaMallocHost(&h->pinned_in, (size_t)n * 2 * kSegment * sizeof(float)));
  CK(cudaMallocHost(&h->pinned_out, (size_t)n * 8 * kSegment * sizeof(float)));
  h->io_cap = n;
}

dmx_status dmx_forward_start(dmx_handle* h, const float* mix, int64_t n, dmx_pending** out) {
  try {
    if (!h || !mix || !out || n <= 0) throw Error(DMX_ERR_INVALID, "dmx_forward_start: bad argument");
    if (h->pending.h) throw Error(DMX_ERR_INVALID, "a forward is already queued on this handle");
    CK(cudaSetDevice(h->device));
    h->launches = 0;
    ensure_io(h, n);
    std::memcpy(h->pinned_in, mix, (size_t)n * 2 * kSegment * sizeof(float));
    CK(cudaMemcpyAsync(h->io_in, h->pinned_in, (size_t)n * 2 * kSegment * sizeof(float),
                       cudaMemcpyHostToDevice, h->stream));
    run_forward(h, h->io_in, n, h->io_out);
    h->mark("end");
    CK(cudaMemcpyAsync(h->pinned_out, h->io_out, (size_t)n * 8 * kSegment * sizeof(float),
                       cudaMemcpyDeviceToHost, h->stream));
    if (!h->pending.done) CK(cudaEventCreateWithFlags(&h->pending.done, cudaEventDisableTiming));
    CK(cudaEventRecord(h->pending.done, h->stream));
    h->pending.h = h;
    h->pending.n = n;
    *out = &h->pending;
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_forward_collect(dmx_pending* p, float* out) {
  try {
    if (!p || !p->h || !out) throw Error(DMX_ERR_INVALID, "dmx_forward_collect: bad argument");
    dmx_handle* h = p->h;
    // bounded wait: poll the event with a deadline instead of blocking forever
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::seconds(600);
    while (true) {
      const cudaError_t e = cudaEventQuery(p->done);
      if (e == cudaSuccess) break;
      if (e != cudaErrorNotReady) CK(e);
      if (std::chrono::steady_clock::now() > deadline) {
        h->pending.h = nullptr;
        throw Error(DMX_ERR_TIMEOUT, "forward did not complete within the deadline");
      }
      std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
    h->pending.h = nullptr;
    check_device_flag(h);
    std::memcpy(out, h->pinned_out, (size_t)p->n * 8 * kSegment * sizeof(float));
    finish_stage_times(h);
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_normalize_track_device(dmx_handle* h, const float* lr_dev, int64_t n,
                                      float* mix_norm_dev, float* mean_std_dev) {
  try {
    if (!h || !lr_dev || !mix_norm_dev || !mean_std_dev || n <= 0)
      throw Error(DMX_ERR_INVALID, "dmx_normalize_track_device: bad argument");
    if ((reinterpret_cast<uintptr_t>(mean_std_dev) & 7) != 0)
      throw Error(DMX_ERR_INVALID, "mean_std_dev must be 8-byte aligned");
    CK(cudaSetDevice(h->device));
    const size_t need = (size_t)track_normalize_scratch_doubles() * sizeof(double);
    if (need > h->norm_cap) {
      cudaFree(h->norm_scratch);
      h->norm_scratch = nullptr;
      h->norm_cap = 0;
      CK(cudaMalloc(&h->norm_scratch, need));
      h->norm_cap = need;
    }
    launch_track_normalize(lr_dev, lr_dev + n, n, h->norm_scratch, mix_norm_dev,
                           reinterpret_cast<float2*>(mean_std_dev), h->stream);
    CK(cudaGetLastError());
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_track_finish(dmx_handle* h, const float* acc_dev, int64_t length,
                            int64_t shift_offset, int64_t max_shift, int segment, double overlap,
                            int shifts, const float* mean_std_dev, float* stems_dev, int64_t t_lo,
                            int64_t t_hi) {
  try {
    if (!h || !acc_dev || !mean_std_dev || !stems_dev || length <= 0)
      throw Error(DMX_ERR_INVALID, "dmx_track_finish: bad argument");
    if (segment != kSegment) throw Error(DMX_ERR_INVALID, "segment must be 343980");
    if (shifts < 0 || shifts > 1)
      throw Error(DMX_ERR_INVALID, "dmx_track_finish handles a single pass (shifts 0 or 1)");
    CK(cudaSetDevice(h->device));
    const int64_t stride = (int64_t)((1.0 - overlap) * (double)segment);
    if (stride <= 0) throw Error(DMX_ERR_INVALID, "overlap leaves a zero stride");
    h->mark("track.finish");
    launch_ola_finish(acc_dev, length, shift_offset, max_shift, segment, stride,
                      h->W(h->m.ola_w.off), reinterpret_cast<const float2*>(mean_std_dev), 1.0f,
                      shifts, nullptr, stems_dev, h->stream, t_lo, t_hi);
    CK(cudaGetLastError());
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

int64_t dmx_num_chunks(int64_t view_length, int segment, double overlap) {
  const int64_t stride = (int64_t)((1.0 - overlap) * (double)segment);
  if (view_length <= 0 || stride <= 0) return 0;
  return (view_length + stride - 1) / stride;
}

}  // extern "C"

namespace {

// The networks of a bag (htdemucs_ft) that run for the requested sources, and
// how their outputs combine (BagCombineForward, api.rs:319-361). A network
// runs only if it carries a nonzero weight on a requested source (api.rs:
// 330-337); for source s the terms are the running networks with a nonzero
// weight on s, in bag order, and their f32 weight sum.
struct BagPlan {
  std::vector<dmx_handle*> nets;  // the networks that run, in bag order
  BagTerms terms{};               // terms.net[][] index `nets`
  cudaEvent_t ev = nullptr;
  ~BagPlan() {
    if (ev) cudaEventDestroy(ev);
  }
};

// Fills t.net / weight / count / total from `weights` (n_nets x sources, row
// per network) and `requested` (sources flags, NULL = all); `slot[k]` is the
// index network k gets in t.out (-1 = it does not run).
BagTerms bag_terms(int n_nets, const float* weights, const int* requested, std::vector<int>* slot) {
  if (n_nets < 1 || n_nets > kBagMaxNets)
    throw Error(DMX_ERR_INVALID, "a bag holds 1 to " + std::to_string(kBagMaxNets) + " networks");
  if (!weights) throw Error(DMX_ERR_INVALID, "bag weights are missing");
  constexpr int S = kBagMaxSources;
  auto req = [&](int s) { return requested == nullptr || requested[s] != 0; };
  BagTerms t{};
  t.sources = S;
  t.channels = 2;
  slot->assign(n_nets, -1);
  int used = 0;
  for (int k = 0; k < n_nets; ++k)
    for (int s = 0; s < S; ++s)
      if (weights[k * S + s] != 0.0f && req(s) && (*slot)[k] < 0) (*slot)[k] = used++;
  for (int s = 0; s < S; ++s) {
    if (!req(s)) continue;
    float total = 0.0f;
    int c = 0;
    for (int k = 0; k < n_nets; ++k) {
      const float w = weights[k * S + s];
      if (w == 0.0f) continue;
      t.net[s][c] = (*slot)[k];
      t.weight[s][c] = w;
      ++c;
      total += w;
    }
    if (total == 0.0f)  // api.rs:355-359
      throw Error(DMX_ERR_INVALID, "no network covers stem index " + std::to_string(s));
    t.count[s] = c;
    t.total[s] = total;
  }
  return t;
}

void make_bag(dmx_handle* const* nets, int n_nets, const float* weights, const int* requested,
              BagPlan* b) {
  if (!nets) throw Error(DMX_ERR_INVALID, "bag networks are missing");
  std::vector<int> slot;
  b->terms = bag_terms(n_nets, weights, requested, &slot);
  for (int k = 0; k < n_nets; ++k) {
    if (slot[k] < 0) continue;
    dmx_handle* hk = nets[k];
    if (!hk) throw Error(DMX_ERR_INVALID, "bag network " + std::to_string(k) + " is NULL");
    if (!b->nets.empty() && hk->device != b->nets[0]->device)
      throw Error(DMX_ERR_INVALID,
                  "the networks of a bag must share one device (for one network per GPU run "
                  "one process per GPU and combine with dmx_bag_combine_device)");
    for (dmx_handle* o : b->nets)
      if (o == hk) throw Error(DMX_ERR_INVALID, "each network of a bag needs its own handle");
    b->nets.push_back(hk);
  }
  if (b->nets.empty())
    throw Error(DMX_ERR_INVALID, "no stem is requested, so no network of the bag would run");
  CK(cudaSetDevice(b->nets[0]->device));
  CK(cudaEventCreateWithFlags(&b->ev, cudaEventDisableTiming));
}

void ensure_bag_out(dmx_handle* h, int64_t G) {
  if (G <= h->bag_cap) return;
  cudaFree(h->bag_out);
  h->bag_out = nullptr;
  h->bag_cap = 0;
  CK(cudaMalloc(&h->bag_out, (size_t)G * 8 * kSegment * sizeof(float)));
  h->bag_cap = G;
}

// BagCombineForward::start (api.rs:326-361) on device: each running network
// forwards the same padded chunks (one after another, ordered by events on
// their streams), then the per-source weighted combination is written to
// `out` on the lead network's stream.
void bag_forward(dmx_handle* lead, BagPlan& b, const float* in, int G, float* out) {
  cudaStream_t prev = lead->stream;
  for (size_t i = 0; i < b.nets.size(); ++i) {
    dmx_handle* hk = b.nets[i];
    CK(cudaSetDevice(hk->device));
    ensure_bag_out(hk, G);
    if (hk->stream != prev) {
      CK(cudaEventRecord(b.ev, prev));
      CK(cudaStreamWaitEvent(hk->stream, b.ev, 0));
    }
    const int64_t before = hk->launches;
    run_forward(hk, in, G, hk->bag_out);
    if (hk != lead) lead->launches += hk->launches - before;
    b.terms.out[i] = hk->bag_out;
    prev = hk->stream;
  }
  if (prev != lead->stream) {
    CK(cudaEventRecord(b.ev, prev));
    CK(cudaStreamWaitEvent(lead->stream, b.ev, 0));
  }
  int64_t reads = 0;
  for (int s = 0; s < b.terms.sources; ++s) reads += b.terms.count[s];
  lead->mark("bag.combine", 0.0, (double)G * 2 * kSegment * 4.0 * (double)(reads + 4));
  launch_bag_combine(b.terms, G, kSegment, out, lead->stream);
  ++lead->launches;
  CK(cudaGetLastError());
}

// Chunks [chunk_lo, chunk_hi) of a shift view: gather, forward (one network,
// or the bag when `bag` is set), overlap-add into acc_dev.
void shard_chunks(dmx_handle* h, BagPlan* bag, const float* mix_norm_dev, int64_t length,
                  int64_t shift_offset, int64_t max_shift, int segment, int64_t stride,
                  int64_t chunk_lo, int64_t chunk_hi, int cap, float* acc_dev, int64_t view_lo,
                  int64_t view_hi) {
  ensure_io(h, cap);
  for (int64_t c0 = chunk_lo; c0 < chunk_hi; c0 += cap) {
    const int G = (int)std::min<int64_t>(cap, chunk_hi - c0);
    h->mark("track.gather");
    launch_gather_chunks(mix_norm_dev, length, shift_offset, max_shift, segment, stride, c0, G,
                         h->io_in, h->stream);
    ++h->launches;
    if (bag)
      bag_forward(h, *bag, h->io_in, G, h->io_out);
    else
      run_forward(h, h->io_in, G, h->io_out);
    h->mark("track.ola");
    launch_ola_accumulate(h->io_out, length, shift_offset, max_shift, segment, stride, c0, G,
                          h->W(h->m.ola_w.off), acc_dev, view_lo, view_hi, h->stream);
    ++h->launches;
    CK(cudaGetLastError());
  }
}

// Pinned host stems that a single-pass separation fills while it runs: after
// each forward batch the output samples that no later chunk touches are
// finished and copied on the handle's copy stream, so the device-to-host
// copy overlaps the remaining forwards (the reference emits frames the same
// way as soon as they are final: streaming.rs:219-260).
struct HostSink {
  float* host = nullptr;  // (8, n) pinned host stems, or
  // blocks of finished stems handed to a callback through two pinned staging
  // buffers: block k is copied while the host hands block k - 1 over and the
  // device already runs the next forward
  dmx_frames_fn emit = nullptr;
  void* user = nullptr;
  int64_t pending_t0 = 0, pending_count = 0;  // the block in flight (count 0: none)
  int pending_slot = 0, next_slot = 0;

  // Waits for the block in flight and hands it over.
  void flush(dmx_handle* h) {
    if (pending_count == 0) return;
    CK(cudaEventSynchronize(h->emit_ev[pending_slot]));
    emit(pending_t0, pending_count, h->emit_pin[pending_slot], user);
    pending_count = 0;
  }
  // Samples [t0, t1) of d_stems (8, n) are final: copy them out as blocks.
  void put(dmx_handle* h, const float* d_stems, int64_t n, int64_t t0, int64_t t1) {
    for (int64_t a = t0; a < t1; a += h->emit_cap) {
      const int64_t count = std::min<int64_t>(h->emit_cap, t1 - a);
      const int slot = next_slot;
      next_slot ^= 1;
      // the slot's previous block was handed over before the block after it was queued
      CK(cudaMemcpy2DAsync(h->emit_pin[slot], (size_t)count * sizeof(float), d_stems + a,
                           (size_t)n * sizeof(float), (size_t)count * sizeof(float), 8,
                           cudaMemcpyDeviceToHost, h->copy_stream));
      CK(cudaEventRecord(h->emit_ev[slot], h->copy_stream));
      flush(h);
      pending_t0 = a;
      pending_count = count;
      pending_slot = slot;
    }
  }
};

// Demucs::separate's device driver for one track (api.rs:438-545, 697-785;
// pipeline.rs:380-515; streaming.rs:52-400) over one network or, with `bag`,
// over the bag's lockstep combination; `h` is the network (the bag's lead)
// whose stream, track workspace and OLA weights the driver uses. With `sink`
// (single pass only) the stems are also copied to the host as they finish.
void separate_track_impl(dmx_handle* h, BagPlan* bag, const float* lr_dev, int64_t n,
                         const dmx_separate_opts* opts, float* d_stems, dmx_progress_fn progress,
                         void* user, HostSink* sink = nullptr) {
  dmx_separate_opts o{1, 0.25, 1.0, 0};
  if (opts) o = *opts;
  if (o.transition_power != 1.0) throw Error(DMX_ERR_INVALID, "transition_power must be 1");
  if (o.shifts < 0) throw Error(DMX_ERR_INVALID, "shifts must be >= 0");
  CK(cudaSetDevice(h->device));
  const int seg = kSegment;
  const int64_t stride = (int64_t)((1.0 - o.overlap) * (double)seg);
  if (stride <= 0) throw Error(DMX_ERR_INVALID, "overlap leaves a zero stride");
  const int64_t max_shift = o.shifts > 0 ? (int64_t)(0.5 * 44100.0) : 0;
  const int64_t view_cap = n + max_shift;
  // track-sized scratch, kept on the handle between calls
  const size_t scratch_bytes = (size_t)track_normalize_scratch_doubles() * sizeof(double);
  const size_t need = (size_t)(2 * n + 8 * view_cap + (o.shifts > 1 ? 8 * n : 0)) * sizeof(float) +
                      scratch_bytes + 512;
  if (need > h->track_cap) {
    cudaFree(h->track_ws);
    h->track_ws = nullptr;
    h->track_cap = 0;
    CK(cudaMalloc(&h->track_ws, need));
    h->track_cap = need;
  }
  double* d_stats = reinterpret_cast<double*>(h->track_ws);
  float2* d_norm = reinterpret_cast<float2*>(h->track_ws + scratch_bytes);
  float* d_mix = reinterpret_cast<float*>(h->track_ws + scratch_bytes + 512);
  float* d_acc = d_mix + 2 * n;
  float* d_pass = o.shifts > 1 ? d_acc + 8 * view_cap : nullptr;
  h->launches = 0;
  if (d_pass) CK(cudaMemsetAsync(d_pass, 0, 8 * n * sizeof(float), h->stream));
  h->mark("track.normalize");
  launch_track_normalize(lr_dev, lr_dev + n, n, d_stats, d_mix, d_norm, h->stream);
  h->launches += 2;
  // ShiftRng (pipeline.rs:136-151), seed 0x5eed1234
  uint64_t rng = 0x5eed1234ULL * 6364136223846793005ULL + 1ULL;
  const int passes = std::max(1, o.shifts);
  const float scale = o.shifts > 0 ? 1.0f / (float)o.shifts : 1.0f;
  size_t done = 0, total = 0;
  std::vector<int64_t> offsets;
  for (int pass = 0; pass < passes; ++pass) {
    int64_t offset = 0;
    if (o.shifts > 0) {
      rng = rng * 6364136223846793005ULL + 1442695040888963407ULL;
      offset = (int64_t)((rng >> 33) % (uint64_t)(max_shift + 1));
    }
    offsets.push_back(offset);
    const int64_t vlen = o.shifts > 0 ? n + max_shift - offset : n;
    total += (size_t)dmx_num_chunks(vlen, seg, o.overlap);
  }
  int max_batch = h->cfg.max_batch;
  if (bag)
    for (dmx_handle* hk : bag->nets) max_batch = std::min(max_batch, hk->cfg.max_batch);
  const int batch = std::max(1, o.batch > 0 ? std::min(o.batch, max_batch) : max_batch);
  // progress counts every running network's chunks (api.rs:764-776)
  const size_t active = bag ? bag->nets.size() : 1;
  const bool stream_out = sink && (sink->host || sink->emit) && passes == 1;
  if (sink && !h->copy_stream) {
    CK(cudaStreamCreateWithFlags(&h->copy_stream, cudaStreamNonBlocking));
    CK(cudaEventCreateWithFlags(&h->copy_ev, cudaEventDisableTiming));
  }
  for (int pass = 0; pass < passes; ++pass) {
    const int64_t offset = offsets[pass];
    const int64_t vlen = o.shifts > 0 ? n + max_shift - offset : n;
    const int64_t chunks = dmx_num_chunks(vlen, seg, o.overlap);
    const int mode = o.shifts == 0 ? 0 : (o.shifts == 1 ? 1 : 2);
    const int64_t trim = o.shifts > 0 ? max_shift - offset : 0;
    int64_t t_done = 0;  // output samples already finished (and copied) by the sink
    CK(cudaMemsetAsync(d_acc, 0, 8 * vlen * sizeof(float), h->stream));
    for (int64_t c0 = 0; c0 < chunks; c0 += batch) {
      const int64_t c1 = std::min<int64_t>(chunks, c0 + batch);
      shard_chunks(h, bag, d_mix, n, offset, max_shift, seg, stride, c0, c1, batch, d_acc, 0, vlen);
      if (stream_out) {
        // view samples below chunk c1's start get no further contribution
        const int64_t t_hi = c1 == chunks ? n : std::min<int64_t>(n, std::max<int64_t>(0, c1 * stride - trim));
        if (t_hi > t_done) {
          h->mark("track.finish");
          ++h->launches;
          launch_ola_finish(d_acc, n, offset, max_shift, seg, stride, h->W(h->m.ola_w.off), d_norm,
                            scale, mode, d_pass, d_stems, h->stream, t_done, t_hi);
          CK(cudaEventRecord(h->copy_ev, h->stream));
          CK(cudaStreamWaitEvent(h->copy_stream, h->copy_ev, 0));
          if (sink->host)
            CK(cudaMemcpy2DAsync(sink->host + t_done, (size_t)n * sizeof(float), d_stems + t_done,
                                 (size_t)n * sizeof(float), (size_t)(t_hi - t_done) * sizeof(float),
                                 8, cudaMemcpyDeviceToHost, h->copy_stream));
          else
            sink->put(h, d_stems, n, t_done, t_hi);
          t_done = t_hi;
        }
      }
      done += (size_t)(c1 - c0);
      if (progress) {
        CK(cudaStreamSynchronize(h->stream));
        progress(done * active, total * active, user);
      }
    }
    if (stream_out) continue;
    h->mark("track.finish");
    ++h->launches;
    launch_ola_finish(d_acc, n, offset, max_shift, seg, stride, h->W(h->m.ola_w.off), d_norm, scale,
                      mode, d_pass, d_stems, h->stream);
  }
  if (o.shifts > 1) ++h->launches;
  if (o.shifts > 1)
    launch_ola_finish(d_acc, n, 0, max_shift, seg, stride, h->W(h->m.ola_w.off), d_norm, scale, 3,
                      d_pass, d_stems, h->stream);
  if (sink && sink->emit) {
    if (!stream_out) {  // several shift passes: every sample is final only now
      CK(cudaEventRecord(h->copy_ev, h->stream));
      CK(cudaStreamWaitEvent(h->copy_stream, h->copy_ev, 0));
      sink->put(h, d_stems, n, 0, n);
    }
    sink->flush(h);
  }
  h->mark("end");
  CK(cudaGetLastError());
}

// Host arrays in, host stems out, through the handle's device staging.
void separate_track_host(dmx_handle* h, BagPlan* bag, const float* left, const float* right,
                         int64_t n, const dmx_separate_opts* opts, float* stems_out,
                         dmx_progress_fn progress, void* user) {
  CK(cudaSetDevice(h->device));
  // host-track staging kept on the handle between calls (grown on demand)
  const size_t need = (size_t)10 * n * sizeof(float);
  if (need > h->host_io_cap) {
    cudaFree(h->host_io);
    h->host_io = nullptr;
    h->host_io_cap = 0;
    CK(cudaMalloc(&h->host_io, need));
    h->host_io_cap = need;
  }
  float* d_lr = h->host_io;
  float* d_stems = h->host_io + 2 * n;
  CK(cudaMemcpyAsync(d_lr, left, n * sizeof(float), cudaMemcpyHostToDevice, h->stream));
  CK(cudaMemcpyAsync(d_lr + n, right, n * sizeof(float), cudaMemcpyHostToDevice, h->stream));
  // pinned stems are copied while the forwards run; pageable ones once at the end (a copy
  // to pageable memory would block this thread before the next forward is enqueued)
  cudaPointerAttributes attr{};
  const bool pinned = cudaPointerGetAttributes(&attr, stems_out) == cudaSuccess &&
                      attr.type == cudaMemoryTypeHost;
  cudaGetLastError();  // a pageable pointer may leave an error behind on some drivers
  const int shifts = opts ? opts->shifts : 1;
  HostSink sink;
  sink.host = stems_out;
  const bool streamed = pinned && shifts <= 1;
  try {
    separate_track_impl(h, bag, d_lr, n, opts, d_stems, progress, user, streamed ? &sink : nullptr);
  } catch (...) {
    if (h->copy_stream) cudaStreamSynchronize(h->copy_stream);  // no copy outlives the call
    throw;
  }
  if (streamed) {
    CK(cudaStreamSynchronize(h->copy_stream));
  } else {
    CK(cudaMemcpyAsync(stems_out, d_stems, 8 * n * sizeof(float), cudaMemcpyDeviceToHost,
                       h->stream));
  }
  CK(cudaStreamSynchronize(h->stream));
  check_device_flag(h);
  if (bag)
    for (dmx_handle* hk : bag->nets)
      if (hk != h) check_device_flag(hk);
  finish_stage_times(h);
}

// Many tracks through one network with their chunks pooled into full
// forwards (the many-track throughput configuration). The work units are (track,
// shift pass, chunk) in that order; consecutive units fill each forward of
// `batch` chunks regardless of which track or pass they belong to. Every
// track is driven exactly as separate_track_impl drives it — its own global
// normalisation, the same ShiftRng offsets (a fresh ShiftRng per track, as
// each Demucs::separate call seeds its own: pipeline.rs:416-418), its own
// overlap-add accumulator and finish — so each track's stems equal
// dmx_separate_track's on that track. A track holds one workspace slot
// (normalised mix, moments, pass sum, accumulator) from the forward that
// takes its first chunk to the one that takes its last.
void separate_batch_impl(dmx_handle* h, const float* const* lr_dev, const int64_t* lengths,
                         int n_tracks, const dmx_separate_opts* opts, float* const* stems_dev,
                         dmx_progress_fn progress, void* user) {
  if (!lr_dev || !lengths || !stems_dev || n_tracks < 1)
    throw Error(DMX_ERR_INVALID, "dmx_separate_batch: bad argument");
  dmx_separate_opts o{1, 0.25, 1.0, 0};
  if (opts) o = *opts;
  if (o.transition_power != 1.0) throw Error(DMX_ERR_INVALID, "transition_power must be 1");
  if (o.shifts < 0) throw Error(DMX_ERR_INVALID, "shifts must be >= 0");
  CK(cudaSetDevice(h->device));
  const int seg = kSegment;
  const int64_t stride = (int64_t)((1.0 - o.overlap) * (double)seg);
  if (stride <= 0) throw Error(DMX_ERR_INVALID, "overlap leaves a zero stride");
  const int64_t max_shift = o.shifts > 0 ? (int64_t)(0.5 * 44100.0) : 0;
  const int passes = std::max(1, o.shifts);
  const float scale = o.shifts > 0 ? 1.0f / (float)o.shifts : 1.0f;
  // ShiftRng (pipeline.rs:136-151), seed 0x5eed1234: the same offsets for every track
  std::vector<int64_t> offsets;
  uint64_t rng = 0x5eed1234ULL * 6364136223846793005ULL + 1ULL;
  for (int pass = 0; pass < passes; ++pass) {
    int64_t offset = 0;
    if (o.shifts > 0) {
      rng = rng * 6364136223846793005ULL + 1442695040888963407ULL;
      offset = (int64_t)((rng >> 33) % (uint64_t)(max_shift + 1));
    }
    offsets.push_back(offset);
  }
  auto view_len = [&](int64_t n, int pass) {
    return o.shifts > 0 ? n + max_shift - offsets[pass] : n;
  };
  std::vector<std::vector<int64_t>> chunks(n_tracks);  // per track, per pass
  std::vector<int64_t> first(n_tracks + 1, 0);         // first unit of each track
  int64_t n_max = 0;
  for (int i = 0; i < n_tracks; ++i) {
    if (lengths[i] <= 0 || !lr_dev[i] || !stems_dev[i])
      throw Error(DMX_ERR_INVALID, "track " + std::to_string(i) + " is empty or has no buffer");
    n_max = std::max(n_max, lengths[i]);
    int64_t units = 0;
    for (int pass = 0; pass < passes; ++pass) {
      chunks[i].push_back(dmx_num_chunks(view_len(lengths[i], pass), seg, o.overlap));
      units += chunks[i].back();
    }
    first[i + 1] = first[i] + units;
  }
  const int64_t total = first[n_tracks];
  const int batch = std::max(1, o.batch > 0 ? std::min(o.batch, h->cfg.max_batch) : h->cfg.max_batch);
  // slots: the most tracks any one forward touches
  int slots = 1;
  for (int64_t u0 = 0, i = 0; u0 < total; u0 += batch) {
    const int64_t u1 = std::min<int64_t>(total, u0 + batch);
    while (first[i + 1] <= u0) ++i;
    int64_t j = i;
    while (j + 1 < n_tracks && first[j + 1] < u1) ++j;
    slots = std::max(slots, (int)(j - i + 1));
  }
  const size_t scratch_bytes = (size_t)track_normalize_scratch_doubles() * sizeof(double);
  const size_t slot_floats = (size_t)(2 * n_max + (o.shifts > 1 ? 8 * n_max : 0) + 8 * (n_max + max_shift));
  const size_t slot_bytes = (scratch_bytes + 512 + slot_floats * sizeof(float) + 255) / 256 * 256;
  if ((size_t)slots * slot_bytes > h->batch_cap) {
    cudaFree(h->batch_ws);
    h->batch_ws = nullptr;
    h->batch_cap = 0;
    CK(cudaMalloc(&h->batch_ws, (size_t)slots * slot_bytes));
    h->batch_cap = (size_t)slots * slot_bytes;
  }
  struct Slot {
    double* stats;
    float2* norm;
    float* mix;
    float* pass;
    float* acc;
  };
  auto slot_at = [&](int k) {
    char* base = h->batch_ws + (size_t)k * slot_bytes;
    Slot sl;
    sl.stats = reinterpret_cast<double*>(base);
    sl.norm = reinterpret_cast<float2*>(base + scratch_bytes);
    sl.mix = reinterpret_cast<float*>(base + scratch_bytes + 512);
    sl.pass = o.shifts > 1 ? sl.mix + 2 * n_max : nullptr;
    sl.acc = sl.mix + 2 * n_max + (o.shifts > 1 ? 8 * n_max : 0);
    return sl;
  };
  std::vector<int> free_slots;
  for (int k = slots - 1; k >= 0; --k) free_slots.push_back(k);
  std::vector<int> slot_of(n_tracks, -1);
  ensure_io(h, batch);
  h->launches = 0;
  const float* w_ola = h->W(h->m.ola_w.off);
  struct Run {
    int track, pass;
    int64_t c0, count, at;  // chunks [c0, c0 + count) of the pass, at forward row `at`
  };
  int ti = 0, tp = 0;
  int64_t tc = 0;  // cursor: next unit is chunk tc of pass tp of track ti
  for (int64_t u0 = 0; u0 < total; u0 += batch) {
    const int G = (int)std::min<int64_t>(batch, total - u0);
    std::vector<Run> runs;
    for (int64_t left = G, at = 0; left > 0;) {
      const int64_t take = std::min<int64_t>(left, chunks[ti][tp] - tc);
      runs.push_back({ti, tp, tc, take, at});
      at += take;
      left -= take;
      tc += take;
      if (tc == chunks[ti][tp]) {
        tc = 0;
        if (++tp == passes) {
          tp = 0;
          ++ti;
        }
      }
    }
    // tracks that start here: a slot, the global normalisation, a cleared pass sum
    for (const Run& r : runs) {
      if (r.pass != 0 || r.c0 != 0) continue;
      const int i = r.track;
      slot_of[i] = free_slots.back();
      free_slots.pop_back();
      const Slot sl = slot_at(slot_of[i]);
      h->mark("track.normalize");
      launch_track_normalize(lr_dev[i], lr_dev[i] + lengths[i], lengths[i], sl.stats, sl.mix,
                             sl.norm, h->stream);
      h->launches += 2;
      if (sl.pass) CK(cudaMemsetAsync(sl.pass, 0, 8 * lengths[i] * sizeof(float), h->stream));
    }
    for (const Run& r : runs) {
      const Slot sl = slot_at(slot_of[r.track]);
      h->mark("track.gather");
      launch_gather_chunks(sl.mix, lengths[r.track], offsets[r.pass], max_shift, seg, stride, r.c0,
                           (int)r.count, h->io_in + r.at * 2 * seg, h->stream);
      ++h->launches;
    }
    run_forward(h, h->io_in, G, h->io_out);
    for (const Run& r : runs) {
      const int i = r.track;
      const Slot sl = slot_at(slot_of[i]);
      const int64_t n = lengths[i];
      const int64_t vlen = view_len(n, r.pass);
      if (r.c0 == 0) CK(cudaMemsetAsync(sl.acc, 0, 8 * vlen * sizeof(float), h->stream));
      h->mark("track.ola");
      launch_ola_accumulate(h->io_out + r.at * 8 * seg, n, offsets[r.pass], max_shift, seg, stride,
                            r.c0, (int)r.count, w_ola, sl.acc, 0, vlen, h->stream);
      ++h->launches;
      if (r.c0 + r.count < chunks[i][r.pass]) continue;
      const int mode = o.shifts == 0 ? 0 : (o.shifts == 1 ? 1 : 2);
      h->mark("track.finish");
      launch_ola_finish(sl.acc, n, offsets[r.pass], max_shift, seg, stride, w_ola, sl.norm, scale,
                        mode, sl.pass, stems_dev[i], h->stream);
      ++h->launches;
      if (r.pass + 1 < passes) continue;
      if (o.shifts > 1) {
        launch_ola_finish(sl.acc, n, 0, max_shift, seg, stride, w_ola, sl.norm, scale, 3, sl.pass,
                          stems_dev[i], h->stream);
        ++h->launches;
      }
      free_slots.push_back(slot_of[i]);
      slot_of[i] = -1;
    }
    CK(cudaGetLastError());
    if (progress) {
      CK(cudaStreamSynchronize(h->stream));
      progress((size_t)(u0 + G), (size_t)total, user);
    }
  }
  h->mark("end");
}

}  // namespace

extern "C" {

dmx_status dmx_separate_track_multi(dmx_handle* const* hs, int n_handles, const float* left,
                                    const float* right, int64_t n, const dmx_separate_opts* opts,
                                    float* stems_out) {
  std::vector<dmx_handle*> H;
  try {
    if (!hs || n_handles < 1 || n_handles > 64 || !left || !right || !stems_out || n <= 0)
      throw Error(DMX_ERR_INVALID, "dmx_separate_track_multi: bad argument");
    for (int k = 0; k < n_handles; ++k) {
      if (!hs[k]) throw Error(DMX_ERR_INVALID, "handle " + std::to_string(k) + " is NULL");
      for (dmx_handle* o : H)
        if (o == hs[k]) throw Error(DMX_ERR_INVALID, "each rank needs its own handle");
      H.push_back(hs[k]);
    }
    dmx_separate_opts o{1, 0.25, 1.0, 0};
    if (opts) o = *opts;
    if (o.transition_power != 1.0) throw Error(DMX_ERR_INVALID, "transition_power must be 1");
    if (o.shifts < 0 || o.shifts > 1)
      throw Error(DMX_ERR_INVALID,
                  "dmx_separate_track_multi runs one pass (shifts 0 or 1); for more shift passes "
                  "use dmx_separate_track or dmx_separate_batch per GPU");
    const int seg = kSegment;
    const int64_t stride = (int64_t)((1.0 - o.overlap) * (double)seg);
    if (stride <= 0) throw Error(DMX_ERR_INVALID, "overlap leaves a zero stride");
    // the single pass's view (ShiftRng's first draw, pipeline.rs:136-151, 416-418)
    const int64_t max_shift = o.shifts > 0 ? (int64_t)(0.5 * 44100.0) : 0;
    int64_t offset = 0;
    if (o.shifts > 0) {
      uint64_t rng = 0x5eed1234ULL * 6364136223846793005ULL + 1ULL;
      rng = rng * 6364136223846793005ULL + 1442695040888963407ULL;
      offset = (int64_t)((rng >> 33) % (uint64_t)(max_shift + 1));
    }
    const int64_t vlen = o.shifts > 0 ? n + max_shift - offset : n;
    const int64_t trim = o.shifts > 0 ? max_shift - offset : 0;
    const int64_t chunks = dmx_num_chunks(vlen, seg, o.overlap);
    const int mode = o.shifts == 0 ? 0 : 1;
    // contiguous chunk ranges, the first `extra` ranks one chunk more
    struct Rank {
      int64_t lo, hi, own_hi, send_lo, send_hi, t_lo, t_hi;
      double* stats;
      float2* norm;
      float *lr, *mix, *acc, *stems;
    };
    std::vector<Rank> R(n_handles);
    const int64_t base = chunks / n_handles, extra = chunks % n_handles;
    int64_t c = 0;
    for (int k = 0; k < n_handles; ++k) {
      Rank& r = R[k];
      r.lo = c;
      r.hi = c + base + (k < extra ? 1 : 0);
      c = r.hi;
      const bool any = r.hi > r.lo;
      const int64_t span_hi = any ? std::min(vlen, (r.hi - 1) * stride + seg) : 0;
      r.own_hi = !any ? 0 : (r.hi == chunks ? vlen : r.hi * stride);
      r.send_lo = r.own_hi;
      r.send_hi = any && r.hi < chunks ? span_hi : r.own_hi;
      const int64_t own_lo = r.lo * stride;
      r.t_lo = any ? std::max<int64_t>(0, own_lo - trim) : 0;
      r.t_hi = any ? std::max(r.t_lo, std::min(n, r.own_hi - trim)) : 0;
    }
    // per rank: the whole track, normalised (deterministic, so every rank agrees), and this
    // rank's chunks overlap-added into a view-sized accumulator
    const size_t scratch_bytes = (size_t)track_normalize_scratch_doubles() * sizeof(double);
    for (int k = 0; k < n_handles; ++k) {
      dmx_handle* h = H[k];
      Rank& r = R[k];
      CK(cudaSetDevice(h->device));
      const size_t need_ws = (size_t)(2 * n + 8 * (n + max_shift)) * sizeof(float) + scratch_bytes + 512;
      if (need_ws > h->track_cap) {
        cudaFree(h->track_ws);
        h->track_ws = nullptr;
        h->track_cap = 0;
        CK(cudaMalloc(&h->track_ws, need_ws));
        h->track_cap = need_ws;
      }
      const size_t need_io = (size_t)10 * n * sizeof(float);
      if (need_io > h->host_io_cap) {
        cudaFree(h->host_io);
        h->host_io = nullptr;
        h->host_io_cap = 0;
        CK(cudaMalloc(&h->host_io, need_io));
        h->host_io_cap = need_io;
      }
      if (!h->shard_done) CK(cudaEventCreateWithFlags(&h->shard_done, cudaEventDisableTiming));
      r.stats = reinterpret_cast<double*>(h->track_ws);
      r.norm = reinterpret_cast<float2*>(h->track_ws + scratch_bytes);
      r.mix = reinterpret_cast<float*>(h->track_ws + scratch_bytes + 512);
      r.acc = r.mix + 2 * n;
      r.lr = h->host_io;
      r.stems = h->host_io + 2 * n;
      h->launches = 0;
      CK(cudaMemcpyAsync(r.lr, left, n * sizeof(float), cudaMemcpyHostToDevice, h->stream));
      CK(cudaMemcpyAsync(r.lr + n, right, n * sizeof(float), cudaMemcpyHostToDevice, h->stream));
      h->mark("track.normalize");
      launch_track_normalize(r.lr, r.lr + n, n, r.stats, r.mix, r.norm, h->stream);
      h->launches += 2;
      CK(cudaMemsetAsync(r.acc, 0, 8 * vlen * sizeof(float), h->stream));
      if (r.hi > r.lo) {
        const int cap = std::max(1, o.batch > 0 ? std::min(o.batch, h->cfg.max_batch) : h->cfg.max_batch);
        shard_chunks(h, nullptr, r.mix, n, offset, max_shift, seg, stride, r.lo, r.hi, cap, r.acc, 0,
                     vlen);
      }
      CK(cudaEventRecord(h->shard_done, h->stream));
    }
    // boundary: rank k + 1 copies rank k's tail (after rank k's chunks) and adds it
    for (int k = 0; k + 1 < n_handles; ++k) {
      const Rank& a = R[k];
      Rank& b = R[k + 1];
      const int64_t w = a.send_hi - a.send_lo;
      if (w <= 0 || b.hi <= b.lo) continue;
      dmx_handle* hb = H[k + 1];
      CK(cudaSetDevice(hb->device));
      const size_t need = (size_t)8 * w * sizeof(float);
      if (need > hb->tail_cap) {
        cudaFree(hb->tail_buf);
        hb->tail_buf = nullptr;
        hb->tail_cap = 0;
        CK(cudaMalloc(&hb->tail_buf, need));
        hb->tail_cap = need;
      }
      CK(cudaStreamWaitEvent(hb->stream, H[k]->shard_done, 0));
      for (int row = 0; row < 8; ++row)
        CK(cudaMemcpyPeerAsync(hb->tail_buf + row * w, hb->device, a.acc + row * vlen + a.send_lo,
                               H[k]->device, (size_t)w * sizeof(float), hb->stream));
      hb->mark("track.merge");
      launch_tail_add(b.acc + a.send_lo, vlen, hb->tail_buf, w, 8, hb->stream);
      ++hb->launches;
      CK(cudaGetLastError());
    }
    // each rank finishes the samples it owns and copies them straight to the host stems
    for (int k = 0; k < n_handles; ++k) {
      dmx_handle* h = H[k];
      const Rank& r = R[k];
      if (r.t_hi <= r.t_lo) continue;
      CK(cudaSetDevice(h->device));
      h->mark("track.finish");
      launch_ola_finish(r.acc, n, offset, max_shift, seg, stride, h->W(h->m.ola_w.off), r.norm, 1.0f,
                        mode, nullptr, r.stems, h->stream, r.t_lo, r.t_hi);
      ++h->launches;
      CK(cudaMemcpy2DAsync(stems_out + r.t_lo, (size_t)n * sizeof(float), r.stems + r.t_lo,
                           (size_t)n * sizeof(float), (size_t)(r.t_hi - r.t_lo) * sizeof(float), 8,
                           cudaMemcpyDeviceToHost, h->stream));
      h->mark("end");
    }
    for (dmx_handle* h : H) {
      CK(cudaSetDevice(h->device));
      CK(cudaStreamSynchronize(h->stream));
      check_device_flag(h);
      finish_stage_times(h);
    }
    return DMX_OK;
  } catch (const Error& e) {
    for (dmx_handle* h : H) {  // no copy into the caller's memory outlives the call
      cudaSetDevice(h->device);
      cudaStreamSynchronize(h->stream);
    }
    return fail(e);
  } catch (const std::exception& e) {
    for (dmx_handle* h : H) {
      cudaSetDevice(h->device);
      cudaStreamSynchronize(h->stream);
    }
    return fail_std(e);
  }
}

dmx_status dmx_separate_batch_device(dmx_handle* h, const float* const* lr_dev,
                                     const int64_t* lengths, int n_tracks,
                                     const dmx_separate_opts* opts, float* const* stems_dev,
                                     dmx_progress_fn progress, void* user) {
  try {
    if (!h) throw Error(DMX_ERR_INVALID, "dmx_separate_batch_device: bad argument");
    separate_batch_impl(h, lr_dev, lengths, n_tracks, opts, stems_dev, progress, user);
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_separate_batch(dmx_handle* h, const float* const* left, const float* const* right,
                              const int64_t* lengths, int n_tracks, const dmx_separate_opts* opts,
                              float* const* stems_out, dmx_progress_fn progress, void* user) {
  try {
    if (!h || !left || !right || !lengths || !stems_out || n_tracks < 1)
      throw Error(DMX_ERR_INVALID, "dmx_separate_batch: bad argument");
    CK(cudaSetDevice(h->device));
    int64_t sum = 0;
    for (int i = 0; i < n_tracks; ++i) {
      if (lengths[i] <= 0 || !left[i] || !right[i] || !stems_out[i])
        throw Error(DMX_ERR_INVALID, "track " + std::to_string(i) + " is empty or has no buffer");
      sum += lengths[i];
    }
    // every track's input (2 n) and stems (8 n) stay on the device for the call
    const size_t need = (size_t)10 * sum * sizeof(float);
    if (need > h->batch_io_cap) {
      cudaFree(h->batch_io);
      h->batch_io = nullptr;
      h->batch_io_cap = 0;
      CK(cudaMalloc(&h->batch_io, need));
      h->batch_io_cap = need;
    }
    std::vector<const float*> d_lr(n_tracks);
    std::vector<float*> d_stems(n_tracks);
    float* at = h->batch_io;
    for (int i = 0; i < n_tracks; ++i) {
      const int64_t n = lengths[i];
      d_lr[i] = at;
      CK(cudaMemcpyAsync(at, left[i], n * sizeof(float), cudaMemcpyHostToDevice, h->stream));
      CK(cudaMemcpyAsync(at + n, right[i], n * sizeof(float), cudaMemcpyHostToDevice, h->stream));
      d_stems[i] = at + 2 * n;
      at += 10 * n;
    }
    separate_batch_impl(h, d_lr.data(), lengths, n_tracks, opts, d_stems.data(), progress, user);
    for (int i = 0; i < n_tracks; ++i)
      CK(cudaMemcpyAsync(stems_out[i], d_stems[i], 8 * lengths[i] * sizeof(float),
                         cudaMemcpyDeviceToHost, h->stream));
    CK(cudaStreamSynchronize(h->stream));
    check_device_flag(h);
    finish_stage_times(h);
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_track_shard(dmx_handle* h, const float* mix_norm_dev, int64_t length,
                           int64_t shift_offset, int64_t max_shift, int segment, double overlap,
                           double transition_power, int64_t chunk_lo, int64_t chunk_hi, int batch,
                           float* acc_dev, int64_t view_lo, int64_t view_hi) {
  try {
    if (segment != kSegment) throw Error(DMX_ERR_INVALID, "segment must be 343980");
    if (transition_power != 1.0) throw Error(DMX_ERR_INVALID, "transition_power must be 1");
    CK(cudaSetDevice(h->device));
    const int64_t stride = (int64_t)((1.0 - overlap) * (double)segment);
    if (stride <= 0) throw Error(DMX_ERR_INVALID, "overlap leaves a zero stride");
    const int cap = std::max(1, batch > 0 ? std::min(batch, h->cfg.max_batch) : h->cfg.max_batch);
    shard_chunks(h, nullptr, mix_norm_dev, length, shift_offset, max_shift, segment, stride, chunk_lo,
                 chunk_hi, cap, acc_dev, view_lo, view_hi);
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_separate_track_device(dmx_handle* h, const float* lr_dev, int64_t n,
                                     const dmx_separate_opts* opts, float* d_stems,
                                     dmx_progress_fn progress, void* user) {
  try {
    if (!h || !lr_dev || !d_stems || n <= 0)
      throw Error(DMX_ERR_INVALID, "dmx_separate_track_device: bad argument");
    separate_track_impl(h, nullptr, lr_dev, n, opts, d_stems, progress, user);
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_bag_combine_device(const float* const* outs_dev, int n_nets, const float* weights,
                                  const int* requested, int64_t n_segments, int64_t samples,
                                  float* combined_dev, void* stream) {
  try {
    if (!outs_dev || !combined_dev || n_segments <= 0 || samples <= 0)
      throw Error(DMX_ERR_INVALID, "dmx_bag_combine_device: bad argument");
    std::vector<int> slot;
    BagTerms t = bag_terms(n_nets, weights, requested, &slot);
    for (int k = 0; k < n_nets; ++k) {
      if (slot[k] < 0) continue;
      if (!outs_dev[k])
        throw Error(DMX_ERR_INVALID, "bag output " + std::to_string(k) + " is NULL but weighted");
      t.out[slot[k]] = outs_dev[k];
    }
    launch_bag_combine(t, n_segments, samples, combined_dev, static_cast<cudaStream_t>(stream));
    CK(cudaGetLastError());
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_bag_forward_device(dmx_handle* const* nets, int n_nets, const float* weights,
                                  const int* requested, const float* mix_dev, int64_t n,
                                  float* out_dev) {
  try {
    if (!mix_dev || !out_dev || n <= 0)
      throw Error(DMX_ERR_INVALID, "dmx_bag_forward_device: bad argument");
    BagPlan bag;
    make_bag(nets, n_nets, weights, requested, &bag);
    dmx_handle* lead = bag.nets[0];
    lead->launches = 0;
    int cap = lead->cfg.max_batch;
    for (dmx_handle* hk : bag.nets) cap = std::min(cap, hk->cfg.max_batch);
    cap = std::max(1, cap);
    for (int64_t s0 = 0; s0 < n; s0 += cap) {
      const int G = (int)std::min<int64_t>(cap, n - s0);
      bag_forward(lead, bag, mix_dev + s0 * 2 * kSegment, G, out_dev + s0 * 8 * kSegment);
    }
    lead->mark("end");
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_separate_track_bag_device(dmx_handle* const* nets, int n_nets, const float* weights,
                                         const int* requested, const float* lr_dev, int64_t n,
                                         const dmx_separate_opts* opts, float* stems_dev,
                                         dmx_progress_fn progress, void* user) {
  try {
    if (!lr_dev || !stems_dev || n <= 0)
      throw Error(DMX_ERR_INVALID, "dmx_separate_track_bag_device: bad argument");
    BagPlan bag;
    make_bag(nets, n_nets, weights, requested, &bag);
    separate_track_impl(bag.nets[0], &bag, lr_dev, n, opts, stems_dev, progress, user);
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_separate_track_bag(dmx_handle* const* nets, int n_nets, const float* weights,
                                  const int* requested, const float* left, const float* right,
                                  int64_t n, const dmx_separate_opts* opts, float* stems_out,
                                  dmx_progress_fn progress, void* user) {
  try {
    if (!left || !right || !stems_out || n <= 0)
      throw Error(DMX_ERR_INVALID, "dmx_separate_track_bag: bad argument");
    BagPlan bag;
    make_bag(nets, n_nets, weights, requested, &bag);
    separate_track_host(bag.nets[0], &bag, left, right, n, opts, stems_out, progress, user);
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_separate_track(dmx_handle* h, const float* left, const float* right, int64_t n,
                              const dmx_separate_opts* opts, float* stems_out,
                              dmx_progress_fn progress, void* user) {
  try {
    if (!h || !left || !right || !stems_out || n <= 0)
      throw Error(DMX_ERR_INVALID, "dmx_separate_track: bad argument");
    separate_track_host(h, nullptr, left, right, n, opts, stems_out, progress, user);
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_separate_track_emit(dmx_handle* h, const float* left, const float* right, int64_t n,
                                   const dmx_separate_opts* opts, dmx_frames_fn on_frames,
                                   dmx_progress_fn progress, void* user) {
  try {
    if (!h || !left || !right || !on_frames || n <= 0)
      throw Error(DMX_ERR_INVALID, "dmx_separate_track_emit: bad argument");
    CK(cudaSetDevice(h->device));
    dmx_separate_opts o{1, 0.25, 1.0, 0};
    if (opts) o = *opts;
    const int64_t stride = (int64_t)((1.0 - o.overlap) * (double)kSegment);
    if (stride <= 0) throw Error(DMX_ERR_INVALID, "overlap leaves a zero stride");
    const int batch = std::max(1, o.batch > 0 ? std::min(o.batch, h->cfg.max_batch) : h->cfg.max_batch);
    // a block holds what one forward finishes: at most `batch` strides plus one segment
    const int64_t cap = std::min<int64_t>(n, (int64_t)batch * stride + kSegment);
    if (cap > h->emit_cap) {
      for (int i = 0; i < 2; ++i) {
        cudaFreeHost(h->emit_pin[i]);
        h->emit_pin[i] = nullptr;
      }
      h->emit_cap = 0;
      for (int i = 0; i < 2; ++i) {
        CK(cudaMallocHost(&h->emit_pin[i], (size_t)8 * cap * sizeof(float)));
        if (!h->emit_ev[i]) CK(cudaEventCreateWithFlags(&h->emit_ev[i], cudaEventDisableTiming));
      }
      h->emit_cap = cap;
    }
    const size_t need = (size_t)10 * n * sizeof(float);
    if (need > h->host_io_cap) {
      cudaFree(h->host_io);
      h->host_io = nullptr;
      h->host_io_cap = 0;
      CK(cudaMalloc(&h->host_io, need));
      h->host_io_cap = need;
    }
    float* d_lr = h->host_io;
    float* d_stems = h->host_io + 2 * n;
    CK(cudaMemcpyAsync(d_lr, left, n * sizeof(float), cudaMemcpyHostToDevice, h->stream));
    CK(cudaMemcpyAsync(d_lr + n, right, n * sizeof(float), cudaMemcpyHostToDevice, h->stream));
    HostSink sink;
    sink.emit = on_frames;
    sink.user = user;
    try {
      separate_track_impl(h, nullptr, d_lr, n, &o, d_stems, progress, user, &sink);
    } catch (...) {
      cudaStreamSynchronize(h->copy_stream);  // no copy into the staging outlives the call
      throw;
    }
    CK(cudaStreamSynchronize(h->stream));
    check_device_flag(h);
    finish_stage_times(h);
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_selftest_wait_timeout(dmx_handle* h, int wait_ms) {
  try {
    if (!h || wait_ms < 1 || wait_ms > 5000)
      throw Error(DMX_ERR_INVALID, "dmx_selftest_wait_timeout: wait_ms must be in [1, 5000]");
    CK(cudaSetDevice(h->device));
    launch_selftest_wait((uint64_t)wait_ms * 1000000ull, kSelftestCode, h->err, h->stream);
    CK(cudaGetLastError());
    CK(cudaStreamSynchronize(h->stream));  // ends: the kernel's wait is bounded
    check_device_flag(h);                  // turns the raised flag into DMX_ERR_TIMEOUT
    throw Error(DMX_ERR_INVALID, "dmx_selftest_wait_timeout: the wait did not report giving up");
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

int dmx_stage_times(dmx_handle* h, const char** names, float* ms, int* counts, double* flops,
                    double* bytes, int cap) {
  if (!h) return 0;
  const int n = std::min<int>(cap, (int)h->stage_names.size());
  for (int i = 0; i < n; ++i) {
    names[i] = h->stage_names[i].c_str();
    ms[i] = h->stage_ms[i];
    if (counts) counts[i] = h->stage_counts[i];
    if (flops) flops[i] = h->stage_flops[i];
    if (bytes) bytes[i] = h->stage_bytes[i];
  }
  return n;
}

dmx_status dmx_set_stage_timing(dmx_handle* h, int on) {
  if (!h) return DMX_ERR_INVALID;
  h->stage_timing = on != 0;
  return DMX_OK;
}

int64_t dmx_kernel_launches(dmx_handle* h) { return h ? h->launches : 0; }

void* dmx_stream(dmx_handle* h) { return h ? static_cast<void*>(h->stream) : nullptr; }

dmx_status dmx_synchronize(dmx_handle* h) {
  try {
    if (!h) throw Error(DMX_ERR_INVALID, "dmx_synchronize: null handle");
    CK(cudaSetDevice(h->device));
    // bounded wait on the handle's stream
    cudaEvent_t e;
    CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    CK(cudaEventRecord(e, h->stream));
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::seconds(600);
    while (true) {
      const cudaError_t q = cudaEventQuery(e);
      if (q == cudaSuccess) break;
      if (q != cudaErrorNotReady) {
        cudaEventDestroy(e);
        CK(q);
      }
      if (std::chrono::steady_clock::now() > deadline) {
        cudaEventDestroy(e);
        throw Error(DMX_ERR_TIMEOUT, "the handle's stream did not drain within the deadline");
      }
      std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
    CK(cudaEventDestroy(e));
    check_device_flag(h);
    finish_stage_times(h);
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  }
}

}  // extern "C"
