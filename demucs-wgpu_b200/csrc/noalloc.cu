// Allocation-free variant of the track normalisation (dmx_normalize_track_noalloc).
//
// Some callers must not allocate device memory at the point where they need
// the track normalised: a real-time audio host (a DAW or plugin processing
// callback may not block, and cudaMalloc/cudaFree can synchronise the whole
// device), or an application that reserved its whole device-memory budget up
// front and cannot afford an unplanned allocation that may fail or fragment.
// They also cannot create a dmx_handle, which allocates its weights and
// workspace. This entry point takes only the caller's input and output
// buffers and keeps its one piece of scratch — the per-block f64 partial sums
// of the moment reduction — in a file-scope device array that every GPU which
// loads the library holds until the process exits.
#include <cstdio>

#include "dmx.h"
#include "kernels.h"

namespace {

constexpr int64_t kSamplesPerBlock = 65536;  // one block of partials per 65,536 samples
constexpr int kMaxBlocks = 8192;             // => at most 536,870,912 samples per channel

// 2 * 8192 doubles = 128 KiB, shared by every call on a device.
static __device__ __align__(256) double g_norm_partials[2 * kMaxBlocks];

thread_local char g_msg[256];

}  // namespace

extern "C" dmx_status dmx_normalize_track_noalloc(const float* lr_dev, int64_t n,
                                                  float* mix_norm_dev, float* mean_std_dev,
                                                  void* stream) {
  if (!lr_dev || !mix_norm_dev || !mean_std_dev) {
    dmx::set_last_error("dmx_normalize_track_noalloc: null pointer argument");
    return DMX_ERR_INVALID;
  }
  if (n < 1 || n > kSamplesPerBlock * kMaxBlocks) {
    snprintf(g_msg, sizeof(g_msg),
             "dmx_normalize_track_noalloc: %lld samples per channel is outside the "
             "allocation-free limit [1, %lld] (about 3 h 22 min at 44.1 kHz); use "
             "dmx_normalize_track_device for longer tracks",
             (long long)n, (long long)(kSamplesPerBlock * kMaxBlocks));
    dmx::set_last_error(g_msg);
    return DMX_ERR_INVALID;
  }
  if ((reinterpret_cast<uintptr_t>(mean_std_dev) & 7) != 0) {
    dmx::set_last_error("dmx_normalize_track_noalloc: mean_std_dev must be 8-byte aligned");
    return DMX_ERR_INVALID;
  }
  // The device address of the file-scope array on the current device (host
  // code only sees a stand-in symbol). Resolved on every call, with the
  // caller's device current, so a device reset or a new primary context
  // never leaves a stale address behind; once the library's module is loaded
  // on the device this allocates nothing. The very first call on a device may
  // load the module, so it should come before any stream capture.
  void* scratch = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&scratch, g_norm_partials);
  if (e != cudaSuccess) {
    snprintf(g_msg, sizeof(g_msg), "dmx_normalize_track_noalloc: cudaGetSymbolAddress failed (%s)",
             cudaGetErrorString(e));
    dmx::set_last_error(g_msg);
    return DMX_ERR_CUDA;
  }
  const int blocks = (int)((n + kSamplesPerBlock - 1) / kSamplesPerBlock);
  // Every block overwrites its own two partials before they are read, so the
  // array needs no clearing between calls.
  dmx::launch_track_normalize_blocks(lr_dev, lr_dev + n, n, blocks,
                                     static_cast<double*>(scratch), mix_norm_dev,
                                     reinterpret_cast<float2*>(mean_std_dev),
                                     static_cast<cudaStream_t>(stream));
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    snprintf(g_msg, sizeof(g_msg), "dmx_normalize_track_noalloc: launch failed (%s)",
             cudaGetErrorString(e));
    dmx::set_last_error(g_msg);
    return DMX_ERR_CUDA;
  }
  return DMX_OK;
}
