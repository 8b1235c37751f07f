// dmx — command-line front end of the B200 backend over the C ABI of
// include/dmx.h (the reference CLI's `demucs separate` and `demucs bench`,
// demucs-cli main.rs:86-128, 313-602, 1126-1190, with `--device cuda[:N]`).
//
//   dmx separate INPUT.wav -o OUT -m CHECKPOINT [--stem S | --two-stems S
//       [--other-method add|minus|none]] [--shifts N] [--overlap F]
//       [--segment SECONDS] [--device cuda[:N]] [--precision tf32|bf16|tf32x3|fp32]
//       [--batch N] [--timings]
//       [--dump-trace DIR]
//   dmx bench -m CHECKPOINT [--repeats N] [--device cuda[:N]] [--precision P]
//   dmx profile INPUT.wav -m CHECKPOINT [--repeats N] [--device ...] [--precision P]
//   dmx wav-copy IN.wav OUT.wav [--stereo] [--window N]   decode a WAV (whole, or in
//       windows of N frames as separate reads it), write it as float32
//
// OUT is a directory (one <stem>.wav per source, float32) or, for a single stem
// or --stem, a file path. WAV input: PCM 16 / 24 / 32-bit, IEEE float 32 / 64-bit and the
// extensible header's 32-bit float (audio.rs:184-360); mono is duplicated to
// stereo; the sample rate must be the model's 44100 Hz. `separate` never holds
// the track: dmx_separate_track_windowed reads the windows it needs from the
// file (WindowedMix, mix.rs:265-360) and hands over each block of finished
// frames, which is written while the device still separates (FloatWavWriter,
// audio.rs:559-670).
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <set>
#include <string>
#include <sys/stat.h>
#include <sys/types.h>
#include <vector>

#include "dmx.h"

namespace {

struct Fail : std::runtime_error {
  using std::runtime_error::runtime_error;
};

// ---------------------------------------------------------------------------
// WAV
// ---------------------------------------------------------------------------
struct Audio {
  int rate = 0;
  int channels = 0;
  int64_t frames = 0;
  std::vector<float> data;  // channel-major: data[c * frames + t]
};

uint32_t le(const unsigned char* p, int n) {
  uint32_t v = 0;
  for (int i = n - 1; i >= 0; --i) v = (v << 8) | p[i];
  return v;
}

// A WAV file read in windows of frames (the reference CLI's WindowedMix over
// probe_audio, mix.rs:265-360): the RIFF chunks are walked once for fmt and
// data (audio.rs:209-274), then each window is decoded where it lies, scaled
// as soundfile scales it (audio.rs:276-313).
struct WavSource {
  std::string path;
  FILE* f = nullptr;
  int tag = -1, channels = 0, bits = 0, rate = 0;
  int64_t frames = 0;
  off_t data_pos = 0;
  std::vector<unsigned char> buf;

  explicit WavSource(const std::string& p) : path(p) {
    f = std::fopen(p.c_str(), "rb");
    if (!f) throw Fail("cannot open " + p);
    unsigned char h[16];
    if (std::fread(h, 1, 12, f) != 12 || std::memcmp(h, "RIFF", 4) || std::memcmp(h + 8, "WAVE", 4)) {
      std::fclose(f);
      f = nullptr;
      throw Fail(p + ": not a RIFF/WAVE file (only uncompressed WAV is supported)");
    }
    fseeko(f, 0, SEEK_END);
    const off_t size = ftello(f);
    off_t data_len = 0;
    bool have_data = false;
    for (off_t pos = 12; pos + 8 <= size;) {
      fseeko(f, pos, SEEK_SET);
      if (std::fread(h, 1, 8, f) != 8) break;
      const uint32_t csize = le(h + 4, 4);
      const off_t body = pos + 8;
      if (!std::memcmp(h, "fmt ", 4)) {
        if (csize < 16 || body + (off_t)csize > size || std::fread(h, 1, 16, f) != 16)
          fail(p + ": truncated fmt chunk");
        tag = (int)le(h, 2);
        channels = (int)le(h + 2, 2);
        rate = (int)le(h + 4, 4);
        bits = (int)le(h + 14, 2);
      } else if (!std::memcmp(h, "data", 4)) {
        data_pos = body;
        data_len = std::min<off_t>(csize, size - body);
        have_data = true;
        if (tag >= 0) break;
      }
      pos = body + csize + (csize & 1);
    }
    if (tag < 0) fail(p + ": missing fmt chunk");
    if (!have_data) fail(p + ": missing data chunk");
    if (channels <= 0) fail(p + ": zero channels");
    const bool ok = (tag == 3 && (bits == 32 || bits == 64)) ||
                    (tag == 1 && (bits == 16 || bits == 24 || bits == 32)) ||
                    (tag == 0xFFFE && bits == 32);
    if (!ok)
      fail(p + ": unsupported WAV format " + std::to_string(tag) + " with " + std::to_string(bits) +
           " bits per sample");
    if (data_len % (bits / 8 * channels))
      fail(p + ": data chunk is not a whole number of " + std::to_string(channels) +
           "-channel frames");
    frames = (int64_t)(data_len / (bits / 8 * channels));
  }
  ~WavSource() {
    if (f) std::fclose(f);
  }
  WavSource(const WavSource&) = delete;
  WavSource& operator=(const WavSource&) = delete;

  [[noreturn]] void fail(const std::string& why) {
    std::fclose(f);
    f = nullptr;
    throw Fail(why);
  }

  // frames [t0, t0 + count) of channel c into out[c][0 .. count)
  void read(int64_t t0, int64_t count, float* const* out) {
    if (t0 < 0 || count < 0 || t0 + count > frames) throw Fail(path + ": read past the end");
    const int bps = bits / 8, bpf = bps * channels;
    buf.resize((size_t)count * bpf);
    if (fseeko(f, data_pos + (off_t)t0 * bpf, SEEK_SET) != 0 ||
        std::fread(buf.data(), 1, buf.size(), f) != buf.size())
      throw Fail(path + ": read failed");
    for (int64_t t = 0; t < count; ++t)
      for (int c = 0; c < channels; ++c) {
        const unsigned char* s = &buf[(size_t)t * bpf + (size_t)c * bps];
        float v;
        if (tag != 1 && bits == 32) {
          const uint32_t u = le(s, 4);
          std::memcpy(&v, &u, 4);
        } else if (bits == 64) {
          uint64_t u = (uint64_t)le(s, 4) | ((uint64_t)le(s + 4, 4) << 32);
          double d;
          std::memcpy(&d, &u, 8);
          v = (float)d;
        } else if (bits == 16) {
          v = (float)(int16_t)le(s, 2) / 32768.0f;
        } else if (bits == 24) {
          const int32_t raw = (int32_t)(le(s, 3) << 8) >> 8;  // sign extension
          v = (float)raw / 8388608.0f;
        } else {
          v = (float)(int32_t)le(s, 4) / 2147483648.0f;
        }
        out[c][t] = v;
      }
  }

  // both channels of the stereo model: mono is duplicated (audio.rs:38-60)
  void read_stereo(int64_t t0, int64_t count, float* left, float* right) {
    float* out[2] = {left, right};
    read(t0, count, out);
    if (channels == 1) std::memcpy(right, left, (size_t)count * sizeof(float));
  }
};

Audio read_wav(const std::string& path) {
  WavSource src(path);
  Audio a;
  a.rate = src.rate;
  a.channels = src.channels;
  a.frames = src.frames;
  a.data.resize((size_t)a.frames * a.channels);
  std::vector<float*> out(a.channels);
  for (int64_t t0 = 0; t0 < a.frames; t0 += 1 << 18) {
    for (int c = 0; c < a.channels; ++c) out[c] = a.data.data() + (size_t)c * a.frames + t0;
    src.read(t0, std::min<int64_t>(1 << 18, a.frames - t0), out.data());
  }
  return a;
}

// IEEE float32 WAV written frame block by frame block; the sizes are patched
// at close (FloatWavWriter, audio.rs:559-670).
struct WavWriter {
  FILE* f = nullptr;
  std::string path;
  int channels = 2;
  uint64_t frames = 0;
  float peak = 0.f;

  WavWriter(const std::string& p, int rate, int ch) : path(p), channels(ch) {
    f = std::fopen(p.c_str(), "wb");
    if (!f) throw Fail("cannot create " + p);
    unsigned char h[44] = {};
    std::memcpy(h, "RIFF", 4);
    std::memcpy(h + 8, "WAVEfmt ", 8);
    put(h + 16, 16, 4);
    put(h + 20, 3, 2);  // IEEE float
    put(h + 22, (uint32_t)ch, 2);
    put(h + 24, (uint32_t)rate, 4);
    put(h + 28, (uint32_t)rate * 4u * ch, 4);
    put(h + 32, 4u * ch, 2);
    put(h + 34, 32, 2);
    std::memcpy(h + 36, "data", 4);
    std::fwrite(h, 1, 44, f);
  }
  static void put(unsigned char* p, uint32_t v, int n) {
    for (int i = 0; i < n; ++i) p[i] = (unsigned char)(v >> (8 * i));
  }
  // frames x channels, interleaved
  void write(const float* interleaved, int64_t count) {
    for (int64_t i = 0; i < count * channels; ++i) peak = std::max(peak, std::fabs(interleaved[i]));
    if (std::fwrite(interleaved, sizeof(float), (size_t)(count * channels), f) !=
        (size_t)(count * channels))
      throw Fail("writing " + path);
    frames += (uint64_t)count;
  }
  void close() {
    const uint64_t bytes = frames * 4u * channels;
    if (bytes > 0xFFFFFFFFull - 36) throw Fail(path + ": WAV larger than 4 GiB");
    unsigned char s[4];
    put(s, (uint32_t)(36 + bytes), 4);
    std::fseek(f, 4, SEEK_SET);
    std::fwrite(s, 1, 4, f);
    put(s, (uint32_t)bytes, 4);
    std::fseek(f, 40, SEEK_SET);
    std::fwrite(s, 1, 4, f);
    std::fclose(f);
    f = nullptr;
  }
};

std::vector<char> read_file(const std::string& path) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) throw Fail("cannot open " + path);
  std::vector<char> b;
  char buf[1 << 16];
  size_t n;
  while ((n = std::fread(buf, 1, sizeof(buf), f)) > 0) b.insert(b.end(), buf, buf + n);
  std::fclose(f);
  return b;
}

void check(dmx_status s, const char* what) {
  if (s != DMX_OK) throw Fail(std::string(what) + ": " + dmx_last_error());
}

// --device cuda[:N] (the reference's `--device` takes cpu / auto / gpu / an
// adapter; this backend runs one CUDA device)
int parse_device(const std::string& spec) {
  if (spec == "cuda" || spec == "gpu" || spec == "auto") return 0;
  if (spec.rfind("cuda:", 0) == 0) return std::atoi(spec.c_str() + 5);
  throw Fail("--device must be cuda or cuda:N, got " + spec);
}

int parse_precision(const std::string& p) {
  if (p == "tf32") return DMX_TF32;
  if (p == "bf16") return DMX_BF16;
  if (p == "tf32x3") return DMX_TF32X3;
  if (p == "fp32") return DMX_FP32;
  throw Fail("--precision must be tf32, bf16, tf32x3 or fp32");
}

const char* kSources[4] = {"drums", "bass", "other", "vocals"};

struct Args {
  std::vector<std::string> pos;
  std::string output, model, stem, two_stems, other_method = "add", device = "cuda",
                                                     precision = "tf32", dump_trace;
  int shifts = 1, batch = 0, repeats = 3, window = 0;
  double overlap = 0.25, segment = 0.0;
  bool timings = false, stereo = false;
};

Args parse(int argc, char** argv, int from) {
  Args a;
  for (int i = from; i < argc; ++i) {
    const std::string k = argv[i];
    auto val = [&]() -> std::string {
      if (i + 1 >= argc) throw Fail(k + " needs a value");
      return argv[++i];
    };
    if (k == "-o" || k == "--output") a.output = val();
    else if (k == "-m" || k == "--model") a.model = val();
    else if (k == "--stem") a.stem = val();
    else if (k == "--two-stems") a.two_stems = val();
    else if (k == "--other-method") a.other_method = val();
    else if (k == "--shifts") a.shifts = std::atoi(val().c_str());
    else if (k == "--overlap") a.overlap = std::atof(val().c_str());
    else if (k == "--segment") a.segment = std::atof(val().c_str());
    else if (k == "--device") a.device = val();
    else if (k == "--precision") a.precision = val();
    else if (k == "--batch") a.batch = std::atoi(val().c_str());
    else if (k == "--repeats") a.repeats = std::atoi(val().c_str());
    else if (k == "--dump-trace") a.dump_trace = val();
    else if (k == "--timings") a.timings = true;
    else if (k == "--stereo") a.stereo = true;
    else if (k == "--window") a.window = std::atoi(val().c_str());
    else if (!k.empty() && k[0] == '-') throw Fail("unknown option " + k);
    else a.pos.push_back(k);
  }
  return a;
}

dmx_handle* load(const Args& a, int max_batch, double* seconds) {
  if (a.model.empty()) throw Fail("-m CHECKPOINT (.th or .safetensors) is required");
  const auto t0 = std::chrono::steady_clock::now();
  const std::vector<char> blob = read_file(a.model);
  dmx_config cfg;
  dmx_default_config(&cfg);
  cfg.precision = parse_precision(a.precision);
  cfg.max_batch = max_batch;
  dmx_handle* h = nullptr;
  check(dmx_create(&cfg, blob.data(), blob.size(), parse_device(a.device), &h), "loading the model");
  *seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  return h;
}

struct EmitState {
  std::vector<WavWriter*> writers;  // per source, or null
  int stem_index = -1;
  WavWriter* companion = nullptr;
  std::string method;
  WavSource* mix = nullptr;
  std::vector<float> frame, raw;
  std::string error;
};

// dmx_read_fn over the input file: the library asks for the windows it needs
int read_frames(int64_t t0, int64_t count, float* left, float* right, void* user) {
  EmitState& st = *static_cast<EmitState*>(user);
  try {
    st.mix->read_stereo(t0, count, left, right);
    return 0;
  } catch (const std::exception& e) {
    st.error = e.what();
    return 1;
  }
}

void on_frames(int64_t t0, int64_t count, const float* block, void* user) {
  EmitState& st = *static_cast<EmitState*>(user);
  if (!st.error.empty()) return;
  try {
    st.frame.resize((size_t)count * 2);
    // block rows: drums L, drums R, bass L, bass R, other L, other R, vocals L, vocals R
    for (int s = 0; s < 4; ++s) {
      if (!st.writers[s]) continue;
      for (int64_t i = 0; i < count; ++i) {
        st.frame[2 * i] = block[(2 * s) * count + i];
        st.frame[2 * i + 1] = block[(2 * s + 1) * count + i];
      }
      st.writers[s]->write(st.frame.data(), count);
    }
    if (st.companion) {
      if (st.method == "minus") {  // the raw mix of the block, read again from the file
        st.raw.resize((size_t)count * 2);
        st.mix->read_stereo(t0, count, st.raw.data(), st.raw.data() + count);
      }
      for (int64_t i = 0; i < count; ++i)
        for (int c = 0; c < 2; ++c) {
          float v = 0.f;
          if (st.method == "add") {
            for (int s = 0; s < 4; ++s)
              if (s != st.stem_index) v += block[(2 * s + c) * count + i];
          } else {  // minus: the raw mix less the stem
            v = st.raw[(size_t)c * count + i] - block[(2 * st.stem_index + c) * count + i];
          }
          st.frame[2 * i + c] = v;
        }
      st.companion->write(st.frame.data(), count);
    }
  } catch (const std::exception& e) {
    st.error = e.what();
  }
}

// --dump-trace: every traced intermediate of the first forward as <name>.npy
// (write_trace, main.rs:735-743; '.', '#' and '/' become '_'). Later forwards
// trace the same names and are skipped.
struct TraceDump {
  std::string dir, error;
  std::set<std::string> seen;
};

void write_npy(const std::string& path, const int64_t* shape, int ndim, const float* data) {
  std::string dims;
  int64_t count = 1;
  for (int i = 0; i < ndim; ++i) {
    dims += std::to_string(shape[i]) + (ndim == 1 || i + 1 < ndim ? "," : "");
    if (i + 1 < ndim) dims += " ";
    count *= shape[i];
  }
  std::string header = "{'descr': '<f4', 'fortran_order': False, 'shape': (" + dims + "), }";
  const size_t total = 10 + header.size() + 1;
  header.append((64 - total % 64) % 64, ' ');
  header += '\n';
  FILE* f = std::fopen(path.c_str(), "wb");
  if (!f) throw Fail("cannot create " + path);
  const unsigned char magic[8] = {0x93, 'N', 'U', 'M', 'P', 'Y', 1, 0};
  const unsigned char hl[2] = {(unsigned char)(header.size() & 255), (unsigned char)(header.size() >> 8)};
  std::fwrite(magic, 1, 8, f);
  std::fwrite(hl, 1, 2, f);
  std::fwrite(header.data(), 1, header.size(), f);
  const size_t wrote = std::fwrite(data, sizeof(float), (size_t)count, f);
  std::fclose(f);
  if (wrote != (size_t)count) throw Fail("writing " + path);
}

void on_trace(const char* name, const float* data, const int64_t* shape, int ndim, void* user) {
  TraceDump& t = *static_cast<TraceDump*>(user);
  if (!t.error.empty() || !t.seen.insert(name).second) return;
  try {
    std::string safe = name;
    for (char& c : safe)
      if (c == '.' || c == '#' || c == '/') c = '_';
    write_npy(t.dir + "/" + safe + ".npy", shape, ndim, data);
  } catch (const std::exception& e) {
    t.error = e.what();
  }
}

// Audio::ensure_channels(2) (audio.rs:38-60): mono is duplicated for the
// stereo model; other channel counts are refused.
void ensure_stereo(Audio& a, const std::string& path) {
  if (a.channels == 1) {
    a.data.insert(a.data.end(), a.data.begin(), a.data.end());
    a.channels = 2;
  } else if (a.channels != 2) {
    throw Fail(path + " has " + std::to_string(a.channels) + " channels; the model is stereo");
  }
}

// WAV in, made stereo, 44100 Hz checked
Audio read_mix(const std::string& path) {
  Audio mix = read_wav(path);
  if (mix.rate != 44100)
    throw Fail(path + " is at " + std::to_string(mix.rate) + " Hz but the model wants 44100 Hz");
  ensure_stereo(mix, path);
  return mix;
}

int cmd_separate(const Args& a) {
  if (a.pos.size() != 1) throw Fail("usage: dmx separate INPUT.wav -o OUT -m CHECKPOINT [options]");
  if (a.output.empty()) throw Fail("-o OUT is required");
  if (!a.stem.empty() && !a.two_stems.empty()) throw Fail("--stem and --two-stems exclude each other");
  WavSource mix(a.pos[0]);
  if (mix.rate != 44100)
    throw Fail(a.pos[0] + " is at " + std::to_string(mix.rate) + " Hz but the model wants 44100 Hz");
  if (mix.channels > 2)
    throw Fail(a.pos[0] + " has " + std::to_string(mix.channels) + " channels; the model is stereo");
  if (mix.frames == 0) throw Fail(a.pos[0] + " holds no samples");
  const std::string named = !a.stem.empty() ? a.stem : a.two_stems;
  int stem_index = -1;
  if (!named.empty()) {
    for (int s = 0; s < 4; ++s)
      if (named == kSources[s]) stem_index = s;
    if (stem_index < 0) throw Fail("--stem/--two-stems must be one of drums, bass, other, vocals");
  }
  const bool companion = !a.two_stems.empty() && a.other_method != "none";
  if (companion && a.other_method != "add" && a.other_method != "minus")
    throw Fail("--other-method must be add, minus or none");
  // An OUT with an extension is one file when no companion is written
  // (main.rs:410-420); four stems cannot share it.
  const size_t slash = a.output.find_last_of('/');
  const std::string leaf = slash == std::string::npos ? a.output : a.output.substr(slash + 1);
  const bool single_file = !companion && leaf.find('.') != std::string::npos && leaf.find('.') > 0;
  if (single_file && stem_index < 0)
    throw Fail("-o " + a.output + " names one file; pick the stem with --stem");
  if (!single_file) mkdir(a.output.c_str(), 0755);
  auto path_for = [&](const std::string& name) {
    return single_file ? a.output : a.output + "/" + name + ".wav";
  };
  const int batch = a.batch > 0 ? a.batch : 16;
  double load_s = 0.0;
  dmx_handle* h = load(a, batch, &load_s);
  EmitState st;
  st.writers.assign(4, nullptr);
  std::vector<std::string> written;
  for (int s = 0; s < 4; ++s)
    if (stem_index < 0 || s == stem_index) st.writers[s] = new WavWriter(path_for(kSources[s]), 44100, 2);
  if (companion) {
    st.companion = new WavWriter(
        path_for((a.other_method == "add" ? "no_" : "minus_") + named), 44100, 2);
    st.method = a.other_method;
  }
  st.stem_index = stem_index;
  st.mix = &mix;
  TraceDump trace;
  if (!a.dump_trace.empty()) {
    mkdir(a.dump_trace.c_str(), 0755);
    trace.dir = a.dump_trace;
    check(dmx_set_trace(h, on_trace, &trace), "tracing");
  }
  dmx_separate_opts o{a.shifts, a.overlap, 1.0, batch, a.segment};
  const auto t0 = std::chrono::steady_clock::now();
  // the track is read window by window, never whole (host or device)
  const dmx_status rc =
      dmx_separate_track_windowed(h, read_frames, mix.frames, &o, on_frames, nullptr, &st);
  const double elapsed = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  const std::string err = !st.error.empty() ? st.error : rc != DMX_OK ? dmx_last_error() : "";
  std::vector<WavWriter*> all = st.writers;
  all.push_back(st.companion);
  std::string list;
  for (WavWriter* w : all) {
    if (!w) continue;
    w->close();
    char peak[64];
    snprintf(peak, sizeof(peak), " (peak %.4f)", w->peak);
    list += (list.empty() ? "" : ", ") + w->path + peak;
    delete w;
  }
  dmx_destroy(h);
  if (!err.empty()) throw Fail("separation: " + err);
  if (!trace.error.empty()) throw Fail("--dump-trace: " + trace.error);
  if (!a.dump_trace.empty())
    std::printf("wrote %zu traced activations to %s\n", trace.seen.size(), a.dump_trace.c_str());
  // report() of main.rs:600-625: the chunk count assumes the default overlap
  const double audio_s = (double)mix.frames / 44100.0;
  std::printf("separation %.2fs for %.3fs -> RTFx %.2fx | + %.2fs load = end-to-end RTFx %.2fx\n",
              elapsed, audio_s, audio_s / elapsed, load_s, audio_s / (elapsed + load_s));
  if (a.timings) {
    const double seg = a.segment > 0 ? a.segment : 7.8;
    const int64_t stride = (int64_t)(0.75 * (double)(int64_t)(44100.0 * seg));
    const double chunks = audio_s * 44100.0 / (double)stride;
    std::printf("per chunk: %.0f ms of model input, %.1fx raw (%.0f chunks)\n",
                elapsed / chunks * 1000.0, seg / (elapsed / chunks), chunks);
  }
  std::printf("wrote %s\n", list.c_str());
  return 0;
}

// `demucs bench` (main.rs:1126-1190): one warm-up, then the mean of `repeats`
// forwards of one segment of LCG noise through the SegmentForward pair.
int cmd_bench(const Args& a) {
  double load_s = 0.0;
  dmx_handle* h = load(a, 1, &load_s);
  std::printf("load %.2fs\n", load_s);
  const int L = 343980;
  std::vector<float> mix(2 * L), out(8 * (size_t)L);
  uint32_t rng = 12345u;
  for (float& v : mix) {
    rng = rng * 1664525u + 1013904223u;
    v = ((float)(rng >> 8) / 8388608.0f - 1.0f) * 0.1f;
  }
  dmx_pending* p = nullptr;
  check(dmx_forward_start(h, mix.data(), 1, &p), "forward");
  check(dmx_forward_collect(p, out.data()), "forward");
  const int repeats = std::max(1, a.repeats);
  const auto t0 = std::chrono::steady_clock::now();
  for (int r = 0; r < repeats; ++r) {
    check(dmx_forward_start(h, mix.data(), 1, &p), "forward");
    check(dmx_forward_collect(p, out.data()), "forward");
  }
  const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() / repeats;
  const double sec = (double)L / 44100.0;
  std::printf("chunk forward %.1f ms for %.3fs of audio -> %.2fx raw (%.1f GB/s of input audio)\n",
              el * 1000.0, sec, sec / el, sec * 2 * 4.0 * 44100.0 / el / 1e9);
  dmx_destroy(h);
  return 0;
}

// `demucs profile` (main.rs:745-790): the first segment of INPUT, globally
// normalised (scan_norm, streaming.rs:52-78) and zero padded, forwarded once
// as a warm-up and then `repeats` times with per-launch device timing; the
// table lists each kernel tag by total time per forward.
int cmd_profile(const Args& a) {
  if (a.pos.size() != 1) throw Fail("usage: dmx profile INPUT.wav -m CHECKPOINT [--repeats N]");
  const Audio mix = read_mix(a.pos[0]);
  double load_s = 0.0;
  dmx_handle* h = load(a, 1, &load_s);
  const int L = 343980;
  double sum = 0.0, sum_sq = 0.0;
  for (int64_t t = 0; t < mix.frames; ++t) {
    const double r = ((double)mix.data[t] + (double)mix.data[mix.frames + t]) / 2.0;
    sum += r;
    sum_sq += r * r;
  }
  const double count = (double)mix.frames;
  const float mean = (float)(sum / count);
  const double var = count > 1.0 ? (sum_sq - sum * sum / count) / (count - 1.0) : 0.0;
  const float std_ = (float)std::sqrt(std::max(var, 0.0)) + 1e-8f;
  std::vector<float> seg(2 * (size_t)L, 0.f), out(8 * (size_t)L);
  const int64_t n = std::min<int64_t>(mix.frames, L);
  for (int c = 0; c < 2; ++c)
    for (int64_t t = 0; t < n; ++t) seg[(size_t)c * L + t] = (mix.data[(size_t)c * mix.frames + t] - mean) / std_;
  std::printf("model loaded in %.2fs | segment %d samples (%.2fs) | %d repeats\n", load_s, L,
              L / 44100.0, std::max(1, a.repeats));
  dmx_pending* p = nullptr;
  check(dmx_forward_start(h, seg.data(), 1, &p), "forward");
  check(dmx_forward_collect(p, out.data()), "forward");
  check(dmx_set_stage_timing(h, 1), "stage timing");
  const int repeats = std::max(1, a.repeats);
  struct Row {
    double ms = 0;
    long calls = 0;
  };
  std::vector<std::pair<std::string, Row>> rows;
  const char* names[256];
  float ms[256];
  int counts[256];
  const auto t0 = std::chrono::steady_clock::now();
  for (int r = 0; r < repeats; ++r) {
    check(dmx_forward_start(h, seg.data(), 1, &p), "forward");
    check(dmx_forward_collect(p, out.data()), "forward");
    const int k = dmx_stage_times(h, names, ms, counts, nullptr, nullptr, 256);
    for (int i = 0; i < k; ++i) {
      auto it = std::find_if(rows.begin(), rows.end(), [&](const auto& e) { return e.first == names[i]; });
      if (it == rows.end()) {
        rows.push_back({names[i], Row{}});
        it = rows.end() - 1;
      }
      it->second.ms += ms[i];
      it->second.calls += counts[i];
    }
  }
  const double wall = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() / repeats;
  dmx_destroy(h);
  std::sort(rows.begin(), rows.end(), [](const auto& x, const auto& y) { return x.second.ms > y.second.ms; });
  std::printf("one segment: %.1f ms wall per forward\n", wall * 1000.0);
  std::printf("%-28s %10s %9s %9s\n", "stage", "total ms", "per call", "calls");
  for (const auto& [name, row] : rows)
    std::printf("%-28s %10.2f %9.3f %9ld\n", name.c_str(), row.ms / repeats,
                row.calls ? row.ms / row.calls : 0.0, row.calls / repeats);
  return 0;
}

// wav-copy: decode and write back as float32. With --window N the input is
// read through WavSource in windows of N frames (with --stereo: the two
// channels separate's read callback hands to the library), the path separate
// uses, instead of whole.
int cmd_wav_copy(const Args& a) {
  if (a.pos.size() != 2) throw Fail("usage: dmx wav-copy IN.wav OUT.wav [--stereo] [--window N]");
  if (a.window > 0) {
    WavSource src(a.pos[0]);
    const int ch = a.stereo ? 2 : src.channels;
    if (a.stereo && src.channels > 2) throw Fail(a.pos[0] + ": more than two channels");
    WavWriter w(a.pos[1], src.rate, ch);
    std::vector<float> cols((size_t)a.window * ch), inter((size_t)a.window * ch);
    for (int64_t t0 = 0; t0 < src.frames; t0 += a.window) {
      const int64_t count = std::min<int64_t>(a.window, src.frames - t0);
      std::vector<float*> out(ch);
      for (int c = 0; c < ch; ++c) out[c] = cols.data() + (size_t)c * count;
      if (a.stereo)
        src.read_stereo(t0, count, out[0], out[1]);
      else
        src.read(t0, count, out.data());
      for (int64_t t = 0; t < count; ++t)
        for (int c = 0; c < ch; ++c) inter[(size_t)t * ch + c] = out[c][t];
      w.write(inter.data(), count);
    }
    w.close();
    std::printf("%d Hz, %d channels, %lld frames\n", src.rate, ch, (long long)src.frames);
    return 0;
  }
  Audio in = read_wav(a.pos[0]);
  if (a.stereo) ensure_stereo(in, a.pos[0]);
  WavWriter w(a.pos[1], in.rate, in.channels);
  std::vector<float> inter((size_t)in.frames * in.channels);
  for (int64_t t = 0; t < in.frames; ++t)
    for (int c = 0; c < in.channels; ++c) inter[(size_t)t * in.channels + c] = in.data[(size_t)c * in.frames + t];
  w.write(inter.data(), in.frames);
  w.close();
  std::printf("%d Hz, %d channels, %lld frames\n", in.rate, in.channels, (long long)in.frames);
  return 0;
}

}  // namespace

int main(int argc, char** argv) {
  try {
    if (argc < 2) throw Fail("usage: dmx separate|bench|profile|wav-copy ...");
    const std::string cmd = argv[1];
    const Args a = parse(argc, argv, 2);
    if (cmd == "separate") return cmd_separate(a);
    if (cmd == "bench") return cmd_bench(a);
    if (cmd == "profile") return cmd_profile(a);
    if (cmd == "wav-copy") return cmd_wav_copy(a);
    throw Fail("unknown command " + cmd + " (separate, bench, profile, wav-copy)");
  } catch (const std::exception& e) {
    std::fprintf(stderr, "dmx: %s\n", e.what());
    return 1;
  }
}
