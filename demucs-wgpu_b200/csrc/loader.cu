// Weight ingestion (dmx_create's host work): the safetensors container
// (safetensors.rs:38-160), the f32 upcast of other dtypes, and the repacking of
// every layer into the layouts the kernels read (weights.rs:211-578 names the
// tensors; the decoder index runs backwards, weights.rs:512-526).
#include <cmath>
#include <cstdio>

#include "runtime.cuh"

namespace dmx {

namespace {

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

}  // namespace

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
  if (n > len - 8) throw Error(DMX_ERR_WEIGHTS, "safetensors header runs past the blob");
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
      // string -> string map; `kwargs` holds the model configuration as JSON
      j.expect('{');
      if (j.peek('}')) {
        j.expect('}');
      } else {
        while (true) {
          const std::string key = j.str();
          j.expect(':');
          if (j.peek('"')) {
            const std::string value = j.str();
            if (key == "kwargs") check_kwargs_json(value);
          } else {
            j.skip();
          }
          if (j.peek(',')) { j.expect(','); continue; }
          j.expect('}');
          break;
        }
      }
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
      // element count and byte size without overflow: a malformed header must
      // not pass the check with a wrapped product
      size_t count = 1;
      for (int64_t d : t.shape) {
        if (d < 0 || (d > 0 && count > data_len / (size_t)d))
          throw Error(DMX_ERR_WEIGHTS, name + ": shape larger than the blob");
        count *= (size_t)d;
      }
      if (count > data_len / (size_t)width || b < a || b > data_len ||
          b - a != count * (size_t)width)
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

namespace {

// fp32 -> nearest tf32 (ties to even), in an fp32 container.
float round_tf32_impl(float x) {
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
                int rows, bool bf16 = false) {
    const HostTensor& w = get(wname, {out, in});
    const HostTensor& b = get(bname, {out});
    Packed p = pack(1, in, rows, false, b.data + row0,
                    [&](int, int ci, int co) { return w.data[(size_t)(row0 + co) * in + ci]; },
                    {{0, 0}});
    if (bf16 && p.has_tc) add_bf16(p, [&](int n, int k) { return w.data[(size_t)(row0 + n) * in + k]; });
    return p;
  }

  // bf16 copy of a packed layer's K-major weights, [Npad][K] (zero rows past N):
  // two bf16 per float slot of the arena, rounded to nearest even.
  template <class F>
  void add_bf16(Packed& p, F value) {
    const size_t count = (size_t)p.Npad * p.K;
    p.bf_off = wb.alloc((count + 1) / 2);
    uint16_t* dst = reinterpret_cast<uint16_t*>(&wb.host[p.bf_off]);
    for (int n = 0; n < p.Npad; ++n)
      for (int k = 0; k < p.K; ++k) {
        const float v = n < p.N ? value(n, k) : 0.0f;
        uint32_t u;
        std::memcpy(&u, &v, 4);
        u += 0x7FFFu + ((u >> 16) & 1u);
        dst[(size_t)n * p.K + k] = (uint16_t)(u >> 16);
      }
    p.has_bf = true;
  }

};

}  // namespace

float round_tf32_host(float x) { return round_tf32_impl(x); }

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
  // The moments of conv2's output for the fused tensor-core DConv kernels:
  // host-side constants v = sum_c w_c, M = sum_c w_c w_c' over conv2's inputs
  // in act order (hidden channels, then the bias input), input i read from K
  // slot slot(i) of the tensor-core copy (high + low parts), then conv1's bias
  // and GroupNorm1's weight and bias.
  auto tc_dconv_moments = [&](int C, DConvLayerW& Lw, auto slot) {
    const int hid = C / 8, act = hid + 1;
    const Packed& p2 = Lw.conv2;
    std::vector<double> w((size_t)2 * C * act);
    for (int n = 0; n < 2 * C; ++n)
      for (int i = 0; i < act; ++i) {
        const size_t e = (size_t)n * p2.K + slot(i);
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
  // The fused tensor-core DConv kernel for C = 48, 96 reads its hidden
  // channels in K slots (dconv_tc_slot): conv1's output rows and conv2's
  // input columns of the tensor-core copies move there.
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
    tc_dconv_moments(C, Lw, [hid](int i) { return dconv_tc_slot(hid, i); });
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
      // C = 192: hidden channel h at K slot h, the bias input at the last slot
      if (C == 192 && Lw.conv1.has_tc && Lw.conv2.has_tc && Lw.conv2.K == 32 &&
          Lw.conv1.Npad >= 32)
        tc_dconv_moments(C, Lw, [hid = C / 8, kb = Lw.conv2.K - 1](int i) { return i < hid ? i : kb; });
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
  // the BF16 build keeps bf16 copies of the transformer linears (kind::f16 GEMMs)
  const bool bf = h->cfg.precision == DMX_BF16;
  for (int s = 0; s < 2; ++s)
    for (int l = 0; l < 5; ++l) {
      LayerW& Lw = s == 0 ? m.layers[l] : m.layers_t[l];
      const std::string at = std::string("crosstransformer.") + (s == 0 ? "layers." : "layers_t.") + std::to_string(l);
      Lw.cross = l % 2 == 1;
      const std::string attn = at + (Lw.cross ? ".cross_attn" : ".self_attn");
      if (Lw.cross) {
        Lw.q = L.linear(attn + ".in_proj_weight", attn + ".in_proj_bias", 1536, 512, 0, 512, bf);
        Lw.kv = L.linear(attn + ".in_proj_weight", attn + ".in_proj_bias", 1536, 512, 512, 1024, bf);
        Lw.n3w = L.vec(at + ".norm3.weight", 512);
        Lw.n3b = L.vec(at + ".norm3.bias", 512);
      } else {
        Lw.qkv = L.linear(attn + ".in_proj_weight", attn + ".in_proj_bias", 1536, 512, 0, 1536, bf);
      }
      Lw.out = L.linear(attn + ".out_proj.weight", attn + ".out_proj.bias", 512, 512, 0, 512, bf);
      Lw.lin1 = L.linear(at + ".linear1.weight", at + ".linear1.bias", 2048, 512, 0, 2048, bf);
      Lw.lin2 = L.linear(at + ".linear2.weight", at + ".linear2.bias", 512, 2048, 0, 512, bf);
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

}  // namespace dmx
