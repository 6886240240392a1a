// ncm_rvq_level_noalloc: one RVQ level with no device allocation at all.
//
// Some callers cannot call cudaMalloc: host plugins whose embedding
// application owns every device allocation (a fixed arena, or a caching
// allocator that must account for all memory), and latency-bound paths that
// may not stall on cudaMalloc, which can synchronise the device. ncm_rvq_level grows the context's workspace with cudaMalloc and
// ncm_ctx_create allocates the context's error word, so neither is usable
// there. This entry point needs no context and allocates nothing: its scratch
// (the bf16 copy of the residual that the tensor cores read, the per-split
// argmin partials, the code norms when the caller passes none, and an error
// word) lives in the file-scope device array below, which every GPU that
// loads the library holds until the process exits.
//
// The array's name is only a host-side stand-in for the device symbol: host
// code must not pass it to a kernel. On the first call on a device, with
// that device current, cudaGetSymbolAddress turns it into the device address
// that is then cached for the device and passed to the kernels. Make that
// first call outside any stream capture. Every call shares the array and
// finds the previous call's contents there, so calls that may overlap on the
// GPU (other streams, other host threads) race on it.
#include <mutex>

#include "internal.h"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;  // 16 MiB per device
constexpr size_t kErrBytes = 256;                          // error word + padding
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_setup_mutex;
void* g_scratch_addr[kMaxDevices] = {};

size_t round256(size_t b) { return (b + 255) & ~static_cast<size_t>(255); }

}  // namespace

extern "C" NCM_API int ncm_rvq_level_noalloc(float* residual, const uint16_t* codebook, const float* sqnorm,
                                             int32_t* codes, int64_t N, int64_t D, int64_t K,
                                             ncm_stream_t stream) {
  using namespace ncm;
  if (N <= 0 || D <= 0 || K <= 0 || N > INT32_MAX || K > INT32_MAX || D > 65536)
    return ncm_fail(NCM_EINVAL, "rvq_level_noalloc: bad shape N=%lld D=%lld K=%lld", (long long)N, (long long)D,
                    (long long)K);
  if (D % 8 != 0) return ncm_fail(NCM_EINVAL, "rvq_level_noalloc: D=%lld must be a multiple of 8", (long long)D);
  if (!residual || !codebook || !codes) return ncm_fail(NCM_EINVAL, "rvq_level_noalloc: null buffer");
  auto misaligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) != 0; };
  if (misaligned(residual) || misaligned(codebook) || misaligned(codes) || (sqnorm && misaligned(sqnorm)))
    return ncm_fail(NCM_EINVAL, "rvq_level_noalloc: buffers must be 16-byte aligned");

  int dev = 0;
  NCM_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return ncm_fail(NCM_EINVAL, "rvq_level_noalloc: device %d unsupported", dev);
  int sms = 0;
  NCM_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));

  // Scratch layout: [error word | bf16 residual copy | split partials | code norms]
  RvqPlan plan = rvq_plan(sms, N, K);
  const size_t shadow_bytes = round256(static_cast<size_t>(N) * D * 2);
  const size_t sq_bytes = sqnorm ? 0 : round256(static_cast<size_t>(K) * sizeof(float));
  size_t need = kErrBytes + shadow_bytes + round256(plan.partial_bytes) + sq_bytes;
  if (need > kNoAllocScratchBytes && plan.splits > 1) {
    // the partials do not fit: one split per row block needs none
    plan.splits = 1;
    plan.tiles_per_split = plan.code_tiles;
    plan.n_units = plan.row_blocks;
    plan.grid = plan.n_units < sms ? plan.n_units : sms;
    plan.partial_bytes = 0;
    need = kErrBytes + shadow_bytes + sq_bytes;
  }
  if (need > kNoAllocScratchBytes)
    return ncm_fail(NCM_EINVAL,
                    "rvq_level_noalloc: N=%lld D=%lld K=%lld needs %zu bytes of scratch; the no-allocation entry "
                    "point has %zu (2*N*D + 4*K must stay below it)",
                    (long long)N, (long long)D, (long long)K, need, kNoAllocScratchBytes);

  void* base = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (g_scratch_addr[dev] == nullptr) {
      void* p = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess || p == nullptr) {
        if (e == cudaSuccess) e = cudaErrorInvalidSymbol;
        return ncm_set_cuda_error(e);
      }
      g_scratch_addr[dev] = p;
    }
    base = g_scratch_addr[dev];
  }
  unsigned char* s = static_cast<unsigned char*>(base);
  int* err = reinterpret_cast<int*>(s);
  uint16_t* shadow = reinterpret_cast<uint16_t*>(s + kErrBytes);
  RvqPartial* part = reinterpret_cast<RvqPartial*>(s + kErrBytes + shadow_bytes);
  float* sq = reinterpret_cast<float*>(s + kErrBytes + shadow_bytes + round256(plan.partial_bytes));

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the error word is the only scratch that must start at zero; the rest is
  // fully written before it is read
  NCM_CUDA_TRY(cudaMemsetAsync(err, 0, sizeof(int), st));
  if (sqnorm == nullptr) {
    NCM_CUDA_TRY(launch_code_sqnorm(codebook, sq, K, D, st));
    sqnorm = sq;
  }
  NCM_CUDA_TRY(launch_f32_to_bf16(residual, shadow, N * D, st));
  CUtensorMap tmA, tmB;
  if (!make_tmap_bf16_2d(&tmA, shadow, N, D, 128) || !make_tmap_bf16_2d(&tmB, codebook, K, D, 256))
    return ncm_fail(NCM_EINVAL, "rvq_level_noalloc: tensor map encoding failed");
  NCM_CUDA_TRY(launch_rvq_argmin(plan, tmA, tmB, sqnorm, codes, part, err, N, D, K, st));
  NCM_CUDA_TRY(
      launch_rvq_apply(plan, part, codes, nullptr, residual, nullptr, codebook, err, N, D, K, true, st));
  return NCM_OK;
}
