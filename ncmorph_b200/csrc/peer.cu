// Peer copies between the GPUs of one node: CUDA IPC mappings of device
// buffers and copy-engine transfers into them.
//
// The row-sharded encode's one exchange is an all-gather of codes and
// reconstructions. Done by NCCL it runs as kernels, which need SMs that the
// persistent distance kernel (one CTA per SM) holds while the exchange
// overlaps the next batch's encode. Done as plain cudaMemcpyAsync between a
// local buffer and a peer's IPC-mapped buffer it runs on the copy engines
// over NVLink and takes no SM. This file provides the plumbing: export a
// buffer's IPC handle (with its offset inside the allocation), map a peer's
// buffer, unmap it, and issue the copies. Synchronisation between ranks is
// the caller's (the Python transport uses two tiny NCCL all-reduces per
// exchange as barriers). No kernel here touches peer memory.
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>
#include <unordered_map>

#include "internal.h"

namespace {

PFN_cuMemGetAddressRange_v3020 address_range_fn() {
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
  });
  return fn;
}

// address returned to the caller -> base that cudaIpcOpenMemHandle mapped
std::mutex g_open_mutex;
std::unordered_map<uintptr_t, void*> g_open;

}  // namespace

extern "C" {

int ncm_ipc_export(const void* dev_ptr, uint64_t bytes, ncm_ipc_handle_t* out) {
  if (dev_ptr == nullptr || out == nullptr || bytes == 0) return ncm_fail(NCM_EINVAL, "ipc_export: bad arguments");
  auto range = address_range_fn();
  if (range == nullptr) return ncm_fail(NCM_ENOTSUP, "ipc_export: cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS)
    return ncm_fail(NCM_EINVAL, "ipc_export: %p is not a device allocation", dev_ptr);
  const uint64_t off = reinterpret_cast<uintptr_t>(dev_ptr) - static_cast<uintptr_t>(base);
  if (off + bytes > size) return ncm_fail(NCM_EINVAL, "ipc_export: %llu bytes run past the allocation",
                                          static_cast<unsigned long long>(bytes));
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return ncm_set_cuda_error(e);
  static_assert(sizeof(h) == sizeof(out->handle), "IPC handle size");
  std::memcpy(out->handle, &h, sizeof(h));
  out->offset = off;
  out->bytes = bytes;
  return NCM_OK;
}

int ncm_ipc_open(const ncm_ipc_handle_t* handle, void** dev_ptr_out) {
  if (handle == nullptr || dev_ptr_out == nullptr) return ncm_fail(NCM_EINVAL, "ipc_open: bad arguments");
  *dev_ptr_out = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle->handle, sizeof(h));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return ncm_set_cuda_error(e);
  void* p = static_cast<uint8_t*>(base) + handle->offset;
  {
    std::lock_guard<std::mutex> lock(g_open_mutex);
    g_open[reinterpret_cast<uintptr_t>(p)] = base;
  }
  *dev_ptr_out = p;
  return NCM_OK;
}

int ncm_ipc_close(void* dev_ptr) {
  void* base = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_open_mutex);
    auto it = g_open.find(reinterpret_cast<uintptr_t>(dev_ptr));
    if (it == g_open.end()) return ncm_fail(NCM_EINVAL, "ipc_close: %p was not returned by ncm_ipc_open", dev_ptr);
    base = it->second;
    g_open.erase(it);
  }
  cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) return ncm_set_cuda_error(e);
  return NCM_OK;
}

int ncm_copy_async(void* dst, const void* src, uint64_t bytes, ncm_stream_t stream) {
  if (bytes == 0) return NCM_OK;
  if (dst == nullptr || src == nullptr) return ncm_fail(NCM_EINVAL, "copy_async: null pointer");
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return ncm_set_cuda_error(e);
  return NCM_OK;
}

int ncm_copy2d_async(void* dst, uint64_t dst_pitch, const void* src, uint64_t src_pitch, uint64_t width_bytes,
                     uint64_t rows, ncm_stream_t stream) {
  if (width_bytes == 0 || rows == 0) return NCM_OK;
  if (dst == nullptr || src == nullptr || dst_pitch < width_bytes || src_pitch < width_bytes)
    return ncm_fail(NCM_EINVAL, "copy2d_async: bad arguments");
  cudaError_t e = cudaMemcpy2DAsync(dst, dst_pitch, src, src_pitch, width_bytes, rows, cudaMemcpyDeviceToDevice,
                                    static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return ncm_set_cuda_error(e);
  return NCM_OK;
}

}  // extern "C"
