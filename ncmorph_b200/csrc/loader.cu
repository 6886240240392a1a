// Device-side safetensors tensor loader (the bf16-native form of
// src/loader.zig:286-345 `read_tensor` + `decode_chunk`): a tensor's bytes
// stream from the file through two pinned staging buffers straight into
// device memory, with the file read of chunk i+1 (four reader threads, one
// slice each) overlapping the host-to-device copy of chunk i. BF16 bytes are stored as they are (no f32
// widening); F16 and F32 are rounded to bf16 on the device with the bf16
// package's rule (packages/bf16/root.zig:17-31: round to nearest even,
// NaN -> 0x7FC0), the operand rounding the bf16 linears apply anyway.
#include <cuda_fp16.h>
#include <fcntl.h>
#include <unistd.h>

#include <cerrno>
#include <cstring>
#include <thread>
#include <vector>

#include "internal.h"

namespace ncm {
namespace {

constexpr size_t kChunk = 16u << 20;  // bytes per staged chunk (a multiple of every element size)
constexpr int kReaders = 4;           // threads reading one chunk, a contiguous slice each

// n bytes at file offset off into h: 0, an errno value, or -1 at an early end of file
int read_slice(int fd, uint8_t* h, size_t n, uint64_t off) {
  size_t got = 0;
  while (got < n) {
    const ssize_t r = pread(fd, h + got, n - got, static_cast<off_t>(off + got));
    if (r < 0 && errno == EINTR) continue;
    if (r < 0) return errno != 0 ? errno : EIO;
    if (r == 0) return -1;
    got += static_cast<size_t>(r);
  }
  return 0;
}

// the chunk split over kReaders threads (one thread below 1 MiB); the first failure is returned
int read_chunk(int fd, uint8_t* h, size_t n, uint64_t off) {
  if (n < (1u << 20)) return read_slice(fd, h, n, off);
  const size_t slice = (n / kReaders + 4095) / 4096 * 4096;
  int res[kReaders] = {0};
  std::vector<std::thread> th;
  for (int r = 1; r < kReaders; ++r) {
    const size_t a = std::min(n, r * slice), b = std::min(n, (r + 1) * slice);
    if (b > a) th.emplace_back([&, r, a, b]() { res[r] = read_slice(fd, h + a, b - a, off + a); });
  }
  res[0] = read_slice(fd, h, std::min(n, slice), off);
  for (auto& t : th) t.join();
  for (int r = 0; r < kReaders; ++r)
    if (res[r] != 0) return res[r];
  return 0;
}

__global__ void __launch_bounds__(256) f16_to_bf16_kernel(const uint16_t* __restrict__ x, uint16_t* __restrict__ y,
                                                          long long n) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  y[i] = f32_to_bf16(__half2float(__ushort_as_half(x[i])));
}

__global__ void __launch_bounds__(256) f32_bits_to_bf16_kernel(const float* __restrict__ x, uint16_t* __restrict__ y,
                                                               long long n) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  y[i] = f32_to_bf16(x[i]);
}

// The context keeps two pinned chunks and their events across calls.
int loader_staging(ncm_ctx* ctx) {
  if (ctx->load_bytes >= kChunk) return NCM_OK;
  for (int b = 0; b < 2; ++b) {
    if (ctx->load_h[b]) cudaFreeHost(ctx->load_h[b]);
    ctx->load_h[b] = nullptr;
    NCM_CUDA_TRY(cudaMallocHost(&ctx->load_h[b], kChunk));
    if (ctx->load_ev[b] == nullptr) NCM_CUDA_TRY(cudaEventCreateWithFlags(&ctx->load_ev[b], cudaEventDisableTiming));
  }
  ctx->load_bytes = kChunk;
  return NCM_OK;
}

int load_ctx_ok(ncm_ctx* ctx) {
  if (ctx == nullptr) return ncm_fail(NCM_EINVAL, "null context");
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev != ctx->device) {
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e != cudaSuccess) return ncm_set_cuda_error(e);
  }
  return NCM_OK;
}

}  // namespace
}  // namespace ncm

using namespace ncm;

extern "C" {

int ncm_load_tensor_bf16(ncm_ctx_t* ctx, const char* path, uint64_t offset, uint64_t nbytes, int32_t dtype,
                         uint16_t* dst, ncm_stream_t stream) {
  int rc = load_ctx_ok(ctx);
  if (rc) return rc;
  if (path == nullptr || dst == nullptr) return ncm_fail(NCM_EINVAL, "load_tensor: null argument");
  int esize;
  switch (dtype) {
    case NCM_DTYPE_BF16: esize = 2; break;
    case NCM_DTYPE_F16: esize = 2; break;
    case NCM_DTYPE_F32: esize = 4; break;
    default: return ncm_fail(NCM_EINVAL, "load_tensor: dtype %d is not BF16, F16 or F32", dtype);
  }
  if (nbytes % esize != 0) return ncm_fail(NCM_EINVAL, "load_tensor: %llu bytes is not a whole number of elements",
                                           (unsigned long long)nbytes);
  if (nbytes == 0) return NCM_OK;
  const int fd = open(path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) return ncm_fail(NCM_EINVAL, "load_tensor: cannot open %s: %s", path, std::strerror(errno));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* dstage = nullptr;
  bool recorded[2] = {false, false};
  auto cleanup = [&]() {
    // the pinned chunks are reused by the next call: let the copies out of them finish
    for (int b = 0; b < 2; ++b)
      if (recorded[b]) cudaEventSynchronize(ctx->load_ev[b]);
    close(fd);
  };
  if ((rc = loader_staging(ctx))) {
    close(fd);
    return rc;
  }
  const size_t chunk = static_cast<size_t>(std::min<uint64_t>(kChunk, nbytes));
  if (dtype != NCM_DTYPE_BF16) {
    dstage = static_cast<uint8_t*>(ctx_workspace(ctx, 2 * chunk));
    if (dstage == nullptr) {
      cleanup();
      return ncm_fail(NCM_ENOMEM, "load_tensor: workspace allocation failed");
    }
  }
  uint64_t done_bytes = 0;
  for (int i = 0; done_bytes < nbytes; ++i) {
    const int b = i & 1;
    const size_t n = static_cast<size_t>(std::min<uint64_t>(chunk, nbytes - done_bytes));
    // staging buffer b is free once the copy (and conversion) issued from it two chunks ago finished
    if (recorded[b]) {
      cudaError_t e = cudaEventSynchronize(ctx->load_ev[b]);
      if (e != cudaSuccess) {
        cleanup();
        return ncm_set_cuda_error(e);
      }
    }
    uint8_t* h = static_cast<uint8_t*>(ctx->load_h[b]);
    const int rerr = read_chunk(fd, h, n, offset + done_bytes);
    if (rerr != 0) {
      cleanup();
      return ncm_fail(NCM_EINVAL, "load_tensor: read of %s in [%llu, %llu) failed: %s", path,
                      (unsigned long long)(offset + done_bytes), (unsigned long long)(offset + done_bytes + n),
                      rerr < 0 ? "unexpected end of file" : std::strerror(rerr));
    }
    cudaError_t e;
    const long long elems = static_cast<long long>(n / esize);
    uint16_t* out = dst + done_bytes / esize;
    if (dtype == NCM_DTYPE_BF16) {
      e = cudaMemcpyAsync(out, h, n, cudaMemcpyHostToDevice, st);
    } else {
      uint8_t* d = dstage + b * chunk;
      e = cudaMemcpyAsync(d, h, n, cudaMemcpyHostToDevice, st);
      if (e == cudaSuccess) {
        Launch _launch(ctx, KID_CAST, st);
        const unsigned blocks = static_cast<unsigned>((elems + 255) / 256);
        if (dtype == NCM_DTYPE_F16)
          f16_to_bf16_kernel<<<blocks, 256, 0, st>>>(reinterpret_cast<const uint16_t*>(d), out, elems);
        else
          f32_bits_to_bf16_kernel<<<blocks, 256, 0, st>>>(reinterpret_cast<const float*>(d), out, elems);
        e = cudaGetLastError();
      }
    }
    if (e == cudaSuccess) e = cudaEventRecord(ctx->load_ev[b], st);
    if (e != cudaSuccess) {
      cleanup();
      return ncm_set_cuda_error(e);
    }
    recorded[b] = true;
    done_bytes += n;
  }
  cleanup();  // returns once the data is on the device
  return NCM_OK;
}

}  // extern "C"
