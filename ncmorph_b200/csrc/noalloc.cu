// ncm_rvq_level_noalloc: one RVQ level with no device allocation at all.
//
// Some callers cannot call cudaMalloc: host plugins whose embedding
// application owns every device allocation (a fixed arena, or a caching
// allocator that must account for all memory), and latency-bound paths that
// may not stall on cudaMalloc, which can synchronise the device. ncm_rvq_level grows the context's workspace with cudaMalloc and
// ncm_ctx_create allocates the context's error word, so neither is usable
// there. This entry point needs no context and allocates nothing: its scratch
// (an error word, the bf16 copy of the residual that the tensor cores read,
// the per-split argmin partials, and the code norms when the caller passes
// none) lives in the file-scope device array below, which every GPU that
// loads the library holds until the process exits.
//
// It runs the same plan and kernels as ncm_rvq_level (CTA pairs for large N,
// the residual update inside the distance kernel for one-split plans, else
// the split merge and update of rvq_apply_kernel), so its codes and residual
// equal that entry point's bit for bit.
//
// The array's name is only a host-side stand-in for the device symbol: host
// code must not pass it to a kernel. The first call in a CUDA context looks
// up the device address with cudaGetSymbolAddress, with that context current,
// and keeps it under the context's unique id (cuCtxGetId), so a host that
// creates its own contexts, or resets the device (which makes a new primary
// context), gets a fresh lookup. Make that first call outside any stream
// capture. Every call shares the array and finds the previous call's contents
// there, so calls that may overlap on the GPU (other streams, other host
// threads) race on it. The error word accumulates device-side failures until
// ncm_rvq_level_noalloc_status reads and clears it.
#include <cudaTypedefs.h>

#include <mutex>

#include "internal.h"
#include "ptx.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;  // 16 MiB per device
constexpr size_t kErrBytes = 256;                          // error word + padding
constexpr int kMaxContexts = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

struct ScratchEntry {
  unsigned long long ctx_id;
  void* addr;
};
std::mutex g_setup_mutex;
ScratchEntry g_scratch[kMaxContexts] = {};
int g_scratch_used = 0;

size_t round256(size_t b) { return (b + 255) & ~static_cast<size_t>(255); }

struct CtxApi {
  PFN_cuCtxGetCurrent_v4000 get_current = nullptr;
  PFN_cuCtxGetId_v12000 get_id = nullptr;
};

const CtxApi& ctx_api() {
  static CtxApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      api.get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      api.get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(p);
  });
  return api;
}

// Device address of the scratch array in the current context (looked up once
// per context). Returns NCM_OK or a failure status.
int scratch_base(void** out) {
  const CtxApi& api = ctx_api();
  CUcontext cu = nullptr;
  unsigned long long id = 0;
  if (api.get_current == nullptr || api.get_id == nullptr || api.get_current(&cu) != CUDA_SUCCESS)
    return ncm_fail(NCM_ECUDA, "rvq_level_noalloc: cannot identify the current CUDA context");
  cudaError_t e;
  if (cu == nullptr) {
    // no context current on this thread yet: make the current device's
    // primary context current (cudaSetDevice initialises it)
    int dev = 0;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess || (e = cudaSetDevice(dev)) != cudaSuccess)
      return ncm_set_cuda_error(e);
    if (api.get_current(&cu) != CUDA_SUCCESS || cu == nullptr)
      return ncm_fail(NCM_ECUDA, "rvq_level_noalloc: no CUDA context is current");
  }
  if (api.get_id(cu, &id) != CUDA_SUCCESS)
    return ncm_fail(NCM_ECUDA, "rvq_level_noalloc: cannot identify the current CUDA context");
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  for (int i = 0; i < g_scratch_used; ++i)
    if (g_scratch[i].ctx_id == id) {
      *out = g_scratch[i].addr;
      return NCM_OK;
    }
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || p == nullptr) {
    if (e == cudaSuccess) e = cudaErrorInvalidSymbol;
    return ncm_set_cuda_error(e);
  }
  if (g_scratch_used < kMaxContexts) {
    g_scratch[g_scratch_used++] = ScratchEntry{id, p};
  } else {
    // a host cycling through more contexts than the table holds: replace the
    // oldest entry (a later call in that context looks its address up again)
    for (int i = 1; i < kMaxContexts; ++i) g_scratch[i - 1] = g_scratch[i];
    g_scratch[kMaxContexts - 1] = ScratchEntry{id, p};
  }
  *out = p;
  return NCM_OK;
}

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
  int sms = 0;
  NCM_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));

  // Scratch layout: [error word | bf16 residual copy | split partials | code norms]
  RvqPlan plan = rvq_plan(sms, N, K, true);
  const size_t shadow_bytes = round256(static_cast<size_t>(N) * D * 2);
  const size_t sq_bytes = sqnorm ? 0 : round256(static_cast<size_t>(K) * sizeof(float));
  size_t need = kErrBytes + shadow_bytes + round256(plan.partial_bytes) + sq_bytes;
  if (need > kNoAllocScratchBytes && plan.splits > 1) {
    // the partials do not fit: one split per 128-row block needs none
    plan.pair = 0;
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
  int rc = scratch_base(&base);
  if (rc) return rc;
  unsigned char* s = static_cast<unsigned char*>(base);
  int* err = reinterpret_cast<int*>(s);
  size_t at = kErrBytes;
  uint16_t* shadow = reinterpret_cast<uint16_t*>(s + at);
  at += shadow_bytes;
  RvqPartial* part = reinterpret_cast<RvqPartial*>(s + at);
  at += round256(plan.partial_bytes);
  float* sq = reinterpret_cast<float*>(s + at);

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the scratch is written before it is read (the error word accumulates)
  if (sqnorm == nullptr) {
    NCM_CUDA_TRY(launch_code_sqnorm(codebook, sq, K, D, st));
    sqnorm = sq;
  }
  NCM_CUDA_TRY(launch_f32_to_bf16(residual, shadow, N * D, st));
  CUtensorMap tmA, tmB;
  if (!make_tmap_bf16_2d(&tmA, shadow, N, D, 128) ||
      !make_tmap_bf16_2d(&tmB, codebook, K, D, rvq_codebook_box_rows(plan)))
    return ncm_fail(NCM_EINVAL, "rvq_level_noalloc: tensor map encoding failed");
  // as in ncm_rvq_level: the residual update runs inside the distance kernel
  // for one-split plans, else rvq_apply_kernel merges the splits and updates
  const RvqFusedUpdate fu{residual, nullptr, nullptr, codebook};
  NCM_CUDA_TRY(launch_rvq_argmin(plan, tmA, tmB, sqnorm, codes, part, err, N, D, K, st,
                                 plan.splits == 1 ? &fu : nullptr));
  if (plan.splits > 1)
    NCM_CUDA_TRY(launch_rvq_apply(plan, part, codes, nullptr, residual, nullptr, codebook, err, N, D, K, true, st));
  return NCM_OK;
}

extern "C" NCM_API int ncm_rvq_level_noalloc_status(ncm_stream_t stream, int32_t* flags) {
  using namespace ncm;
  if (flags != nullptr) *flags = 0;
  void* base = nullptr;
  int rc = scratch_base(&base);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int word = 0;
  NCM_CUDA_TRY(cudaMemcpyAsync(&word, base, sizeof(int), cudaMemcpyDeviceToHost, st));
  NCM_CUDA_TRY(cudaStreamSynchronize(st));
  if (flags != nullptr) *flags = word;
  if (word == 0) return NCM_OK;
  NCM_CUDA_TRY(cudaMemsetAsync(base, 0, sizeof(int), st));
  NCM_CUDA_TRY(cudaStreamSynchronize(st));
  if (word & kErrWaitTimeout)
    return ncm_fail(NCM_ETIMEOUT, "rvq_level_noalloc: a device-side wait timed out (flags %d)", word);
  return ncm_fail(NCM_ERANGE, "rvq_level_noalloc: a kernel met an out-of-range index (flags %d)", word);
}
