// Internal declarations of the host runtime shared by its translation units:
//   loader.cu  — safetensors parsing, weight repacking (dmx_create's work)
//   forward.cu — the handle's launch helpers and the segment forward
//   track.cu   — the separation drivers (one track, many tracks, bags, several GPUs)
//   abi.cu     — the C ABI of include/dmx.h
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "conv_gemm.cuh"
#include "dmx.h"
#include "kernels.h"
#include "tc_gemm.cuh"

namespace dmx {

struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

#define CK(call)                                                                       \
  do {                                                                                 \
    cudaError_t e_ = (call);                                                           \
    if (e_ != cudaSuccess)                                                             \
      throw ::dmx::Error(e_ == cudaErrorMemoryAllocation ? DMX_ERR_NOMEM : DMX_ERR_CUDA, \
                         std::string(#call) + ": " + cudaGetErrorString(e_));          \
  } while (0)

// ---------------------------------------------------------------------------
// Weights (loader.cu)
// ---------------------------------------------------------------------------
struct HostTensor {
  std::vector<int64_t> shape;
  const float* data = nullptr;                // into the blob (F32) or into `owned`
  std::shared_ptr<std::vector<float>> owned;  // the f32 copy of a tensor stored in another dtype
  size_t count() const {
    size_t n = 1;
    for (int64_t s : shape) n *= (size_t)s;
    return n;
  }
};

// Parses and validates a safetensors blob (8-byte little-endian header size,
// JSON header, raw data); every tensor comes back as f32. Its
// __metadata__["kwargs"] is checked with check_kwargs_json.
std::map<std::string, HostTensor> parse_safetensors(const void* blob, size_t len);
// Upcasts n elements of a safetensors dtype ("F16", "BF16", "F64", "I64", ...) to f32.
std::vector<float> decode_tensor(const char* raw, size_t n, const std::string& dtype);
// ckpt.cu: a torch.save zip's state dict as f32 tensors (its kwargs checked).
bool is_torch_zip(const void* blob, size_t len);
std::map<std::string, HostTensor> parse_torch_zip(const void* blob, size_t len);
// Either container, by its first bytes.
std::map<std::string, HostTensor> parse_checkpoint(const void* blob, size_t len);
// Rejects model kwargs (a JSON object) of an architecture other than the
// htdemucs default the kernels implement (DMX_ERR_INVALID naming the field).
void check_kwargs_json(const std::string& text);

constexpr int kBK = 16, kBN = 64;

struct Tap {
  int dy, dx;  // input offset of the tap
};

struct Packed {
  size_t w_off = 0, b_off = 0;  // float offsets into the weight arena
  size_t tc_off = 0;            // K-major copy [Npad][K], rounded to nearest tf32
  size_t tc_lo_off = 0;         // its residual w - tf32(w) (3xTF32 split)
  size_t bf_off = 0;            // bf16 copy [Npad][K], round to nearest even (BF16 build)
  bool has_tc = false;
  bool has_bf = false;
  int cin = 0;       // input channels as packed (zero rows pad it to a multiple of 16)
  int cin_real = 0;  // the layer's own input channels (for the work count)
  double flop_scale = 1.0;  // algorithmic share of the packed K (structural zeros excluded)
  int K = 0, Kpad = 0, N = 0, Npad = 0;
  std::vector<Tap> taps;
  // thin first convolutions (K <= 32, 48 outputs): [K][48] then the bias, in
  // host memory, for the kernel that takes them as a launch parameter
  std::vector<float> host_w;
};

struct Vec {  // a plain per-channel vector on the device
  size_t off = 0;
  int n = 0;
};

struct EncW {
  Packed conv, rewrite;
  int cin = 0, cout = 0;
};

struct DecW {
  Packed rewrite;
  Packed convt[4];   // per output phase
  Packed convt_all;  // the four phases side by side (one GEMM over the input positions)
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
  Vec ola_w;   // triangular transition weight (segment), transition_power 1
  size_t tw_off = 0;  // float2 twiddles (2048)
};

struct DConvLayerW {
  Packed conv1, conv2;
  Vec n1w, n1b, n2w, n2b, gamma;
  std::vector<float> zq;  // the fused tensor-core kernel's moment constants (host memory)
  size_t zq_off = 0;      // the SIMT kernels' moment constants (weight arena)
};

struct DConvFull {
  DConvLayerW layer[2];
  int C = 0, hidden = 0;
};

// fp32 -> nearest tf32 (ties to even), in an fp32 container.
float round_tf32_host(float x);

}  // namespace dmx

// ---------------------------------------------------------------------------
// The handle.
// ---------------------------------------------------------------------------

// One queued dmx_forward_start: its own pinned and device staging, so a
// second forward can be queued while the first is still in flight (the
// reference's queue-one-ahead loop, pipeline.rs:178-190 / streaming.rs:341-383).
struct dmx_pending {
  dmx_handle* h = nullptr;
  bool busy = false;
  int64_t n = 0;
  uint64_t seq = 0;  // order of the starts
  cudaEvent_t done = nullptr;
  float* in_dev = nullptr;
  float* out_dev = nullptr;
  float* pin_in = nullptr;
  float* pin_out = nullptr;
  int64_t cap = 0;  // segments the staging holds
};

constexpr int kPendingSlots = 2;

struct dmx_handle {
  dmx_config cfg{};
  int device = 0;
  cudaStream_t stream = nullptr;
  float* wdev = nullptr;
  dmx::Model m;
  dmx::DConvFull enc_dc[4], tenc_dc[4], dec_dc[4], tdec_dc[4];
  // workspace
  char* ws = nullptr;
  size_t ws_cap = 0, ws_off = 0;
  bool measuring = false;
  size_t ws_peak = 0;
  int64_t launches = 0;
  // device staging of the drivers' chunk batches
  float* io_in = nullptr;
  float* io_out = nullptr;
  int64_t io_cap = 0;
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
  dmx_pending pending[kPendingSlots];
  uint64_t pending_seq = 0;
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
  float* ola_w_custom = nullptr;  // transition weight of a non-default segment / power
  int ola_w_len = 0;
  double ola_w_power = 1.0;
  // dmx_separate_track_windowed: device window, accumulators and output blocks,
  // and the pinned staging its read callback fills
  char* win_ws = nullptr;
  size_t win_cap = 0;
  float* win_pin[2] = {nullptr, nullptr};
  cudaEvent_t win_ev[2] = {nullptr, nullptr};  // the copy that last read win_pin[i]
  cudaEvent_t out_ev[2] = {nullptr, nullptr};  // the copy that last read output block i
  int64_t win_pin_cap = 0;                     // floats per pinned window buffer

  float* W(size_t off) const { return wdev + off; }

  void* alloc(size_t bytes) {
    bytes = (bytes + 255) / 256 * 256;
    if (measuring) {
      ws_off += bytes;
      ws_peak = std::max(ws_peak, ws_off);
      return reinterpret_cast<void*>(0x100);
    }
    if (ws_off + bytes > ws_cap) throw dmx::Error(DMX_ERR_NOMEM, "workspace exhausted");
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

  // Launch helpers (forward.cu).
  void gemm(const dmx::ConvParams& p, int pro, int epi, const char* tag = "gemm",
            const dmx::Packed* pk = nullptr);
  // The tensor-core path alone, for launches the SIMT kernel cannot express
  // (split output columns): false, with nothing launched, when the
  // tensor-core kernel does not take it; the caller then issues another form.
  bool gemm_tc(const dmx::ConvParams& p, int epi, const char* tag, const dmx::Packed& pk);
  bool try_tc(const dmx::ConvParams& p, int pro, int epi, const dmx::Packed& pk);
  bool build_tc(const dmx::ConvParams& p, const dmx::Packed& pk, dmx::TcOperandA& a,
                dmx::TcParams& t);

  void after(const char* what) {
    if (!live()) return;
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
      throw dmx::Error(DMX_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  }
};

namespace dmx {

// Grows a device buffer kept on the handle (frees the old one first; the
// free waits for the device, so no queued work still reads it).
template <class T>
void grow(T*& p, size_t& cap, size_t bytes) {
  if (bytes <= cap) return;
  cudaFree(p);
  p = nullptr;
  cap = 0;
  void* q = nullptr;
  CK(cudaMalloc(&q, bytes));
  p = static_cast<T*>(q);
  cap = bytes;
}

// ---------------------------------------------------------------------------
// forward.cu
// ---------------------------------------------------------------------------
// The whole forward of G segments: mix (G, 2, L) device, normalised chunks ->
// out (G, 4, 2, L) device (Htdemucs::forward, host.rs:202-520).
void forward(dmx_handle* h, const float* mix, int G, float* out);
// Sizes the workspace for `G` segments by a dry run of the launch sequence.
void ensure_workspace(dmx_handle* h, int G);
// n segments in forwards of at most max_batch.
void run_forward(dmx_handle* h, const float* mix_dev, int64_t n, float* out_dev);
// Raises DMX_ERR_TIMEOUT when a tensor-core kernel gave up a bounded wait.
void check_device_flag(dmx_handle* h);
void finish_stage_times(dmx_handle* h);
// Device staging of the drivers' chunk batches (io_in / io_out) for n segments.
void ensure_io(dmx_handle* h, int64_t n);
constexpr int kSelftestCode = 99;  // the error code dmx_selftest_wait_timeout's kernel raises

// ---------------------------------------------------------------------------
// loader.cu
// ---------------------------------------------------------------------------
void load_model(dmx_handle* h, const std::map<std::string, HostTensor>& t);

// ---------------------------------------------------------------------------
// track.cu
// ---------------------------------------------------------------------------
// The offsets ShiftRng(0x5eed_1234) draws for `passes` passes, each in
// [0, max_shift] (pipeline.rs:136-151, 416-418).
std::vector<int64_t> shift_offsets(int passes, int64_t max_shift);

// Split-pass geometry of a separation: the samples the chunks are cut to
// (the model's segment unless overridden), the stride and the transition
// weight.
struct PassGeom {
  int chunk;            // samples per chunk (<= the model's segment)
  int64_t stride;
  const float* weight;  // device, `chunk` floats
};
// Chunk samples of a separation: int(44100 * opts.segment), or the model's
// segment when opts.segment is 0 (streaming.rs:315-316).
int64_t chunk_samples(const dmx_separate_opts& o);
PassGeom pass_geom(dmx_handle* h, int64_t chunk, double overlap, double transition_power);
// Validates and fills the defaults of a dmx_separate_opts.
dmx_separate_opts separate_opts(const dmx_separate_opts* opts);

// The networks of a bag (htdemucs_ft) that run for the requested sources, and
// how their outputs combine (BagCombineForward, api.rs:319-361).
struct BagPlan {
  std::vector<dmx_handle*> nets;  // the networks that run, in bag order
  BagTerms terms{};               // terms.net[][] index `nets`
  cudaEvent_t ev = nullptr;
  ~BagPlan() {
    if (ev) cudaEventDestroy(ev);
  }
};
BagTerms bag_terms(int n_nets, const float* weights, const int* requested, std::vector<int>* slot);
void make_bag(dmx_handle* const* nets, int n_nets, const float* weights, const int* requested,
              BagPlan* b);
void bag_forward(dmx_handle* lead, BagPlan& b, const float* in, int G, float* out);
void shard_chunks(dmx_handle* h, BagPlan* bag, const float* mix_norm_dev, int64_t length,
                  int64_t shift_offset, int64_t max_shift, const PassGeom& pg, int64_t chunk_lo,
                  int64_t chunk_hi, int cap, float* acc_dev, int64_t view_lo, int64_t view_hi);

// Pinned host stems or an emit callback that a single-pass separation fills
// while it runs.
struct HostSink {
  float* host = nullptr;  // (8, n) pinned host stems, or
  // blocks of finished stems handed to a callback through two pinned staging
  // buffers: block k is copied while the host hands block k - 1 over and the
  // device already runs the next forward
  dmx_frames_fn emit = nullptr;
  void* user = nullptr;
  int64_t pending_t0 = 0, pending_count = 0;  // the block in flight (count 0: none)
  int pending_slot = 0, next_slot = 0;
  void flush(dmx_handle* h);
  // samples [t0, t1) of 8 device rows `ld` apart whose column 0 is sample col0
  void put(dmx_handle* h, const float* d_stems, int64_t ld, int64_t t0, int64_t t1,
           int64_t col0 = 0);
};

void ensure_emit(dmx_handle* h, int64_t cap);

void separate_track_impl(dmx_handle* h, BagPlan* bag, const float* lr_dev, int64_t n,
                         const dmx_separate_opts* opts, float* d_stems, dmx_progress_fn progress,
                         void* user, HostSink* sink = nullptr);
void separate_track_host(dmx_handle* h, BagPlan* bag, const float* left, const float* right,
                         int64_t n, const dmx_separate_opts* opts, float* stems_out,
                         dmx_progress_fn progress, void* user);
void separate_batch_impl(dmx_handle* h, const float* const* lr_dev, const int64_t* lengths,
                         int n_tracks, const dmx_separate_opts* opts, float* const* stems_dev,
                         dmx_progress_fn progress, void* user);
void separate_windowed_impl(dmx_handle* h, dmx_read_fn read, int64_t n,
                             const dmx_separate_opts* opts, dmx_frames_fn on_frames,
                             dmx_progress_fn progress, void* user);
void separate_track_multi_impl(const std::vector<dmx_handle*>& H, const float* left,
                               const float* right, int64_t n, const dmx_separate_opts* opts,
                               float* stems_out);

// ---------------------------------------------------------------------------
// abi.cu
// ---------------------------------------------------------------------------
int fail(const Error& e);
int fail_std(const std::exception& e);

}  // namespace dmx
