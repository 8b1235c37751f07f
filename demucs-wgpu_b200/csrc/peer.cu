// Peer memory for one process per GPU on one node: a rank exports a device
// buffer as a CUDA IPC handle, the other ranks map it into their own address
// space, and the overlap-add boundary merge and the stem gather become SM
// loads over NVLink straight from the neighbour's accumulator and stems
// (dmx_rows_add / dmx_rows_copy on the handle's stream). This is the
// multi-process counterpart of dmx_separate_track_multi's peer copies; the
// ordering between ranks comes from the caller (a collective on the same
// streams before and after the reads).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "runtime.cuh"

using namespace dmx;

namespace {

// Base of the cudaMalloc allocation holding `ptr` (an IPC handle names a whole
// allocation; a caching allocator hands out pieces of larger blocks).
CUdeviceptr allocation_base(const void* ptr) {
  using Fn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  static Fn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<Fn>(p);
  });
  if (!fn) throw Error(DMX_ERR_CUDA, "cuMemGetAddressRange is not available");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    throw Error(DMX_ERR_INVALID, "not a device allocation of this process");
  return base;
}

void rows_op(bool add, dmx_handle* h, float* dst, int64_t dst_ld, const float* src, int64_t src_ld,
             int rows, int64_t width) {
  if (!h || !dst || !src || rows < 0 || rows > 65535 || width < 0 || dst_ld < width || src_ld < width)
    throw Error(DMX_ERR_INVALID, add ? "dmx_rows_add: bad argument" : "dmx_rows_copy: bad argument");
  CK(cudaSetDevice(h->device));
  launch_rows(add, dst, dst_ld, src, src_ld, rows, width, h->stream);
  CK(cudaGetLastError());
}

}  // namespace

extern "C" {

dmx_status dmx_ipc_export(int device, const void* dev_ptr, unsigned char handle[64],
                          int64_t* offset) {
  try {
    if (!dev_ptr || !handle || !offset) throw Error(DMX_ERR_INVALID, "dmx_ipc_export: bad argument");
    CK(cudaSetDevice(device));
    const CUdeviceptr base = allocation_base(dev_ptr);
    cudaIpcMemHandle_t h;
    CK(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
    std::memcpy(handle, &h, sizeof(h) < 64 ? sizeof(h) : 64);
    *offset = (int64_t)(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_ipc_open(int device, const unsigned char handle[64], int64_t offset, void** ptr) {
  try {
    if (!handle || !ptr || offset < 0) throw Error(DMX_ERR_INVALID, "dmx_ipc_open: bad argument");
    CK(cudaSetDevice(device));
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void* base = nullptr;
    CK(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
    *ptr = static_cast<char*>(base) + offset;
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_ipc_close(int device, void* ptr, int64_t offset) {
  try {
    if (!ptr || offset < 0) throw Error(DMX_ERR_INVALID, "dmx_ipc_close: bad argument");
    CK(cudaSetDevice(device));
    CK(cudaIpcCloseMemHandle(static_cast<char*>(ptr) - offset));
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_rows_copy(dmx_handle* h, float* dst, int64_t dst_ld, const float* src,
                         int64_t src_ld, int rows, int64_t width) {
  try {
    rows_op(false, h, dst, dst_ld, src, src_ld, rows, width);
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

dmx_status dmx_rows_add(dmx_handle* h, float* dst, int64_t dst_ld, const float* src,
                        int64_t src_ld, int rows, int64_t width) {
  try {
    rows_op(true, h, dst, dst_ld, src, src_ld, rows, width);
    return DMX_OK;
  } catch (const Error& e) {
    return fail(e);
  } catch (const std::exception& e) {
    return fail_std(e);
  }
}

}  // extern "C"
