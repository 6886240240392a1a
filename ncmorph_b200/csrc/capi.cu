// C-ABI entry points of libncm_cuda.so (declared in include/ncm_cuda.h):
// argument validation, context/workspace management and the composition of
// the kernels in rvq.cu and gemm.cu into the reference-shaped operations.
#include <cudaTypedefs.h>

#include <algorithm>
#include <vector>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "internal.h"
#include "ptx.cuh"

namespace {

thread_local char g_last_error[512] = "";

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

PFN_cuTensorMapEncodeTiled_v12000 tmap_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int check_ctx(ncm_ctx* ctx) {
  if (ctx == nullptr) return ncm_fail(NCM_EINVAL, "null context");
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev != ctx->device) {
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e != cudaSuccess) return ncm_set_cuda_error(e);
  }
  return NCM_OK;
}

}  // namespace

int ncm_set_cuda_error(cudaError_t e) {
  std::snprintf(g_last_error, sizeof(g_last_error), "CUDA error %d: %s", static_cast<int>(e), cudaGetErrorString(e));
  return NCM_ECUDA;
}

int ncm_fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

namespace ncm {

const char* const kKernelNames[KID_COUNT] = {"rvq_argmin", "rvq_apply",    "linear_bf16", "rvq_decode",
                                             "code_sqnorm", "pool_avg",     "scale_update", "cast",
                                             "attention",   "decoder_elementwise", "conv_k3",
                                             "upsample"};

Launch::Launch(ncm_ctx* ctx, KernelId id, cudaStream_t stream) : ctx_(ctx), id_(id), stream_(stream) {
  ProfState& p = ctx->prof;
  ++p.launches[id];
  if (!p.on) return;
  auto& v = p.events[id];
  if (p.used[id] == v.size()) {
    cudaEvent_t a = nullptr, b = nullptr;
    if (cudaEventCreate(&a) != cudaSuccess || cudaEventCreate(&b) != cudaSuccess) {
      cudaGetLastError();
      return;
    }
    v.emplace_back(a, b);
  }
  cudaEventRecord(v[p.used[id]].first, stream);
  stop_ = v[p.used[id]].second;
  ++p.used[id];
}

Launch::~Launch() {
  if (stop_ != nullptr) cudaEventRecord(stop_, stream_);
}

void* ctx_workspace(ncm_ctx* ctx, size_t bytes) {
  if (bytes <= ctx->ws_bytes) return ctx->ws;
  if (ctx->ws != nullptr) {
    cudaDeviceSynchronize();
    cudaFree(ctx->ws);
    ctx->ws = nullptr;
    ctx->ws_bytes = 0;
  }
  const size_t want = bytes + bytes / 4;
  if (cudaMalloc(&ctx->ws, want) != cudaSuccess) {
    cudaGetLastError();
    ctx->ws = nullptr;
    return nullptr;
  }
  ctx->ws_bytes = want;
  return ctx->ws;
}

int* rvq_counters(ncm_ctx* ctx, int64_t row_blocks) {
  if (row_blocks <= ctx->rvq_counter_len) return ctx->rvq_counters;
  if (ctx->rvq_counters != nullptr) {
    cudaDeviceSynchronize();
    cudaFree(ctx->rvq_counters);
    ctx->rvq_counters = nullptr;
    ctx->rvq_counter_len = 0;
  }
  const int64_t n = std::max<int64_t>(row_blocks, 4096);
  if (cudaMalloc(&ctx->rvq_counters, sizeof(int) * n) != cudaSuccess ||
      cudaMemset(ctx->rvq_counters, 0, sizeof(int) * n) != cudaSuccess) {
    cudaGetLastError();
    if (ctx->rvq_counters) cudaFree(ctx->rvq_counters);
    ctx->rvq_counters = nullptr;
    return nullptr;
  }
  ctx->rvq_counter_len = n;
  return ctx->rvq_counters;
}

bool make_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  return make_tmap_bf16_2d_strided(map, base, rows, cols, cols, box_rows);
}

bool make_tmap_bf16_2d_strided(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                               uint64_t row_stride, uint32_t box_rows) {
  auto fn = tmap_encode_fn();
  if (fn == nullptr || rows == 0 || cols == 0 || row_stride < cols || (row_stride * 2) % 16 != 0 || !aligned16(base))
    return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride * 2)};
  cuuint32_t box[2] = {64u, box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// One RVQ level on a bf16 view `a_bf16` of the residual. `resid` is updated
// in place (or initialised from src_bf16 when given); `shadow` receives
// bf16(resid) for the next level when non-null.
static int rvq_level_core(ncm_ctx* ctx, const uint16_t* a_bf16, const uint16_t* src_bf16, float* resid,
                          uint16_t* shadow, const uint16_t* codebook, const float* sqnorm, int32_t* codes,
                          RvqPartial* part, const RvqPlan& plan, int64_t N, int64_t D, int64_t K, bool update,
                          cudaStream_t stream, const RvqTop2* top2 = nullptr) {
  CUtensorMap tmA, tmB;
  if (!make_tmap_bf16_2d(&tmA, a_bf16, N, D, 128) ||
      !make_tmap_bf16_2d(&tmB, codebook, K, D, rvq_codebook_box_rows(plan)))
    return ncm_fail(NCM_EINVAL, "rvq: tensor map encoding failed (N=%lld D=%lld K=%lld)", (long long)N,
                    (long long)D, (long long)K);
  // Code splits merge inside the distance kernel (split fixup) only when no
  // update follows: the CTA finishing a row block's last split writes its
  // codes. With an update, rvq_apply_kernel merges and updates over every SM
  // (the update at the end of the distance kernel measured slower at every
  // split size, whether one CTA or all of a row block's CTAs ran it).
  const bool fixup = plan.splits > 1 && top2 == nullptr && !update;
  int* counters = fixup ? rvq_counters(ctx, plan.row_blocks) : nullptr;
  const bool merged = plan.splits == 1 || counters != nullptr;
  const bool fused = update && merged;
  RvqFusedUpdate fu{resid, src_bf16, shadow, codebook};
  {
    Launch _launch(ctx, KID_RVQ_ARGMIN, stream);
    NCM_CUDA_TRY(launch_rvq_argmin(plan, tmA, tmB, sqnorm, codes, part, ctx->d_err, N, D, K, stream,
                                   fused ? &fu : nullptr, top2, nullptr, counters));
  }
  if (!merged || (update && !fused)) {
    Launch _launch(ctx, KID_RVQ_APPLY, stream);
    NCM_CUDA_TRY(launch_rvq_apply(plan, part, codes, src_bf16, resid, shadow, codebook, ctx->d_err, N, D, K, update,
                                  stream, top2));
  }
  return NCM_OK;
}

// L levels over bf16 rows x with every buffer supplied: resid (f32 [N,D]),
// shadow (bf16 [N,D]), part (split partials). The last level updates resid
// only when keep_resid.
static int rvq_encode_core(ncm_ctx* ctx, const uint16_t* x, const uint16_t* codebooks, const float* sqnorms, int L,
                           int32_t* codes, uint16_t* recon, float* resid, bool keep_resid, uint16_t* shadow,
                           RvqPartial* part, const RvqPlan& plan, int64_t N, int64_t D, int64_t K,
                           cudaStream_t st) {
  RvqLevelsPlan lp;
  if (rvq_levels_plan(ctx->num_sms, N, D, K, L, &lp)) {
    // few row blocks: every level in one launch (clusters share the code range)
    {
      Launch _launch(ctx, KID_RVQ_ARGMIN, st);
      NCM_CUDA_TRY(launch_rvq_levels(lp, x, codebooks, sqnorms, L, codes, resid, keep_resid, shadow, recon,
                                     ctx->d_err, N, D, K, st));
    }
    if (recon != nullptr && !lp.reg) {
      Launch _launch(ctx, KID_DECODE, st);
      NCM_CUDA_TRY(launch_rvq_decode(codes, codebooks, L, recon, nullptr, N, D, K, ctx->d_err, st));
    }
    return NCM_OK;
  }
  for (int l = 0; l < L; ++l) {
    const bool last = (l == L - 1);
    const bool update = !last || keep_resid;
    const uint16_t* a = (l == 0) ? x : shadow;
    int rc = rvq_level_core(ctx, a, l == 0 ? x : nullptr, resid, last ? nullptr : shadow,
                            codebooks + static_cast<size_t>(l) * K * D, sqnorms + static_cast<size_t>(l) * K,
                            codes + static_cast<size_t>(l) * N, part, plan, N, D, K, update, st);
    if (rc) return rc;
  }
  if (recon != nullptr) {
    Launch _launch(ctx, KID_DECODE, st);
    NCM_CUDA_TRY(launch_rvq_decode(codes, codebooks, L, recon, nullptr, N, D, K, ctx->d_err, st));
  }
  return NCM_OK;
}

}  // namespace ncm

using namespace ncm;

extern "C" {

int ncm_version(void) { return 100; }

const char* ncm_status_string(int s) {
  switch (s) {
    case NCM_OK: return "ok";
    case NCM_EINVAL: return "invalid argument";
    case NCM_ECUDA: return "CUDA error";
    case NCM_ENOMEM: return "out of device memory";
    case NCM_ETIMEOUT: return "device wait timed out";
    case NCM_ERANGE: return "index out of range";
    case NCM_ENOTSUP: return "unsupported device";
    default: return "unknown status";
  }
}

const char* ncm_last_error(void) { return g_last_error; }

int ncm_ctx_create(int device, ncm_ctx_t** out) {
  if (out == nullptr) return ncm_fail(NCM_EINVAL, "null output pointer");
  *out = nullptr;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) return ncm_set_cuda_error(e);
  if (device < 0 || device >= n) return ncm_fail(NCM_EINVAL, "device %d out of range (%d devices)", device, n);
  cudaDeviceProp prop;
  NCM_CUDA_TRY(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10 || prop.minor != 0)
    return ncm_fail(NCM_ENOTSUP, "device %d is sm_%d%d; this library is built for sm_100a", device, prop.major,
                    prop.minor);
  NCM_CUDA_TRY(cudaSetDevice(device));
  ncm_ctx* ctx = new ncm_ctx();
  ctx->device = device;
  ctx->num_sms = prop.multiProcessorCount;
  e = cudaMalloc(&ctx->d_err, 256);
  if (e != cudaSuccess) {
    delete ctx;
    return ncm_set_cuda_error(e);
  }
  cudaMemset(ctx->d_err, 0, 256);
  cudaDeviceSynchronize();
  *out = ctx;
  return NCM_OK;
}

int ncm_ctx_destroy(ncm_ctx_t* ctx) {
  if (ctx == nullptr) return NCM_OK;
  cudaSetDevice(ctx->device);
  cudaDeviceSynchronize();
  comm_release(ctx);
  if (ctx->rvq_counters) cudaFree(ctx->rvq_counters);
  if (ctx->kpart) cudaFree(ctx->kpart);
  for (int i = 0; i < 2; ++i) {
    if (ctx->load_h[i]) cudaFreeHost(ctx->load_h[i]);
    if (ctx->load_ev[i]) cudaEventDestroy(ctx->load_ev[i]);
  }
  if (ctx->ws) cudaFree(ctx->ws);
  if (ctx->d_err) cudaFree(ctx->d_err);
  if (ctx->h_stage) cudaFreeHost(ctx->h_stage);
  if (ctx->rope_cos) cudaFree(ctx->rope_cos);
  if (ctx->rope_sin) cudaFree(ctx->rope_sin);
  if (ctx->rope_cos_bf) cudaFree(ctx->rope_cos_bf);
  if (ctx->rope_sin_bf) cudaFree(ctx->rope_sin_bf);
  if (ctx->rope_row_level) cudaFree(ctx->rope_row_level);
  if (ctx->copy_in) cudaStreamDestroy(ctx->copy_in);
  if (ctx->copy_out) cudaStreamDestroy(ctx->copy_out);
  for (int i = 0; i < 2; ++i) {
    if (ctx->ev_in[i]) cudaEventDestroy(ctx->ev_in[i]);
    if (ctx->ev_done[i]) cudaEventDestroy(ctx->ev_done[i]);
    if (ctx->ev_out[i]) cudaEventDestroy(ctx->ev_out[i]);
  }
  delete ctx;
  return NCM_OK;
}

int ncm_sync(ncm_ctx_t* ctx, ncm_stream_t stream) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  NCM_CUDA_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  int err = 0;
  NCM_CUDA_TRY(cudaMemcpy(&err, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (err != 0) {
    cudaMemset(ctx->d_err, 0, sizeof(int));
    // an aborted distance kernel may have left split-fixup counters mid-count
    if ((err & kErrWaitTimeout) && ctx->rvq_counters)
      cudaMemset(ctx->rvq_counters, 0, sizeof(int) * ctx->rvq_counter_len);
    cudaDeviceSynchronize();
    if (err & kErrWaitTimeout) return ncm_fail(NCM_ETIMEOUT, "a device-side pipeline wait timed out (flags %d)", err);
    return ncm_fail(NCM_ERANGE, "a kernel met an out-of-range index (flags %d)", err);
  }
  return NCM_OK;
}

int ncm_f32_to_bf16(ncm_ctx_t* ctx, const float* x, uint16_t* y, int64_t n, ncm_stream_t stream) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if (n < 0 || (n > 0 && (x == nullptr || y == nullptr))) return ncm_fail(NCM_EINVAL, "f32_to_bf16: bad arguments");
  if (!aligned16(x) || !aligned16(y)) return ncm_fail(NCM_EINVAL, "f32_to_bf16: buffers must be 16-byte aligned");
  {
    Launch _launch(ctx, KID_CAST, static_cast<cudaStream_t>(stream));
    NCM_CUDA_TRY(launch_f32_to_bf16(x, y, n, static_cast<cudaStream_t>(stream)));
  }
  return NCM_OK;
}

int ncm_bf16_to_f32(ncm_ctx_t* ctx, const uint16_t* x, float* y, int64_t n, ncm_stream_t stream) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if (n < 0 || (n > 0 && (x == nullptr || y == nullptr))) return ncm_fail(NCM_EINVAL, "bf16_to_f32: bad arguments");
  if (!aligned16(x) || !aligned16(y)) return ncm_fail(NCM_EINVAL, "bf16_to_f32: buffers must be 16-byte aligned");
  {
    Launch _launch(ctx, KID_CAST, static_cast<cudaStream_t>(stream));
    NCM_CUDA_TRY(launch_bf16_to_f32(x, y, n, static_cast<cudaStream_t>(stream)));
  }
  return NCM_OK;
}

int ncm_linear_bf16(ncm_ctx_t* ctx, const uint16_t* x, const uint16_t* w, const uint16_t* bias, uint16_t* y,
                    int64_t M, int64_t K, int64_t N, ncm_stream_t stream) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if (M <= 0 || K <= 0 || N <= 0 || M > INT32_MAX || N > INT32_MAX || K > INT32_MAX)
    return ncm_fail(NCM_EINVAL, "linear: bad shape M=%lld K=%lld N=%lld", (long long)M, (long long)K, (long long)N);
  if (K % 8 != 0) return ncm_fail(NCM_EINVAL, "linear: K=%lld must be a multiple of 8", (long long)K);
  if (!x || !w || !y) return ncm_fail(NCM_EINVAL, "linear: null buffer");
  if (!aligned16(x) || !aligned16(w) || !aligned16(y) || (bias && !aligned16(bias)))
    return ncm_fail(NCM_EINVAL, "linear: buffers must be 16-byte aligned");
  return linear_bf16(ctx, x, w, bias, y, nullptr, M, K, N, static_cast<cudaStream_t>(stream));
}

// Shared body of the host-slice linears: round f32 operands to bf16 on the
// device, run the tensor-core GEMM, copy the result back.
static int linear_host_common(ncm_ctx* ctx, const float* x, const float* w, const float* bias, float* y, int64_t M,
                              int64_t K, int64_t N, bool round_output) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if (M <= 0 || K <= 0 || N <= 0 || M > INT32_MAX || N > INT32_MAX || K > INT32_MAX)
    return ncm_fail(NCM_EINVAL, "linear: bad shape M=%lld K=%lld N=%lld", (long long)M, (long long)K, (long long)N);
  if (!x || !w || !y) return ncm_fail(NCM_EINVAL, "linear: null buffer");
  // Pad K to a multiple of 8 with zeros (TMA rows must be 16-byte strided).
  const int64_t Kp = (K + 7) / 8 * 8;
  WsCarver cv;
  const size_t o_xf = cv.take(sizeof(float) * M * Kp);
  const size_t o_wf = cv.take(sizeof(float) * N * Kp);
  const size_t o_xb = cv.take(2 * M * Kp);
  const size_t o_wb = cv.take(2 * N * Kp);
  const size_t o_bf = cv.take(sizeof(float) * N);
  const size_t o_bb = cv.take(2 * N);
  const size_t o_y = cv.take(sizeof(float) * M * N);
  const size_t o_yb = cv.take(2 * M * N);
  uint8_t* ws = static_cast<uint8_t*>(ctx_workspace(ctx, cv.offset));
  if (ws == nullptr) return ncm_fail(NCM_ENOMEM, "linear: workspace allocation failed");
  float* xf = reinterpret_cast<float*>(ws + o_xf);
  float* wf = reinterpret_cast<float*>(ws + o_wf);
  uint16_t* xb = reinterpret_cast<uint16_t*>(ws + o_xb);
  uint16_t* wb = reinterpret_cast<uint16_t*>(ws + o_wb);
  float* bf = reinterpret_cast<float*>(ws + o_bf);
  uint16_t* bb = reinterpret_cast<uint16_t*>(ws + o_bb);
  float* yf = reinterpret_cast<float*>(ws + o_y);
  uint16_t* yb = reinterpret_cast<uint16_t*>(ws + o_yb);
  cudaStream_t st = 0;
  if (Kp == K) {
    NCM_CUDA_TRY(cudaMemcpyAsync(xf, x, sizeof(float) * M * K, cudaMemcpyHostToDevice, st));
    NCM_CUDA_TRY(cudaMemcpyAsync(wf, w, sizeof(float) * N * K, cudaMemcpyHostToDevice, st));
  } else {
    NCM_CUDA_TRY(cudaMemsetAsync(xf, 0, sizeof(float) * M * Kp, st));
    NCM_CUDA_TRY(cudaMemsetAsync(wf, 0, sizeof(float) * N * Kp, st));
    NCM_CUDA_TRY(cudaMemcpy2DAsync(xf, sizeof(float) * Kp, x, sizeof(float) * K, sizeof(float) * K, M,
                                   cudaMemcpyHostToDevice, st));
    NCM_CUDA_TRY(cudaMemcpy2DAsync(wf, sizeof(float) * Kp, w, sizeof(float) * K, sizeof(float) * K, N,
                                   cudaMemcpyHostToDevice, st));
  }
  {
    Launch _launch(ctx, KID_CAST, st);
    NCM_CUDA_TRY(launch_f32_to_bf16(xf, xb, M * Kp, st));
  }
  {
    Launch _launch(ctx, KID_CAST, st);
    NCM_CUDA_TRY(launch_f32_to_bf16(wf, wb, N * Kp, st));
  }
  const uint16_t* bias_dev = nullptr;
  if (bias != nullptr) {
    NCM_CUDA_TRY(cudaMemcpyAsync(bf, bias, sizeof(float) * N, cudaMemcpyHostToDevice, st));
    {
      Launch _launch(ctx, KID_CAST, st);
      NCM_CUDA_TRY(launch_f32_to_bf16(bf, bb, N, st));
    }
    bias_dev = bb;
  }
  if (round_output) {
    rc = linear_bf16(ctx, xb, wb, bias_dev, yb, nullptr, M, Kp, N, st);
    if (rc) return rc;
    {
      Launch _launch(ctx, KID_CAST, st);
      NCM_CUDA_TRY(launch_bf16_to_f32(yb, yf, M * N, st));
    }
  } else {
    rc = linear_bf16(ctx, xb, wb, bias_dev, nullptr, yf, M, Kp, N, st);
    if (rc) return rc;
  }
  NCM_CUDA_TRY(cudaMemcpyAsync(y, yf, sizeof(float) * M * N, cudaMemcpyDeviceToHost, st));
  return ncm_sync(ctx, st);
}

int ncm_linear_bf16_host_f32(ncm_ctx_t* ctx, const float* x, const float* w, const float* bias, float* y, int64_t M,
                             int64_t K, int64_t N) {
  return linear_host_common(ctx, x, w, bias, y, M, K, N, true);
}

int ncm_matmul_host_f32(ncm_ctx_t* ctx, const float* x, const float* w, float* y, int64_t M, int64_t K, int64_t N) {
  return linear_host_common(ctx, x, w, nullptr, y, M, K, N, false);
}

int ncm_code_sqnorm(ncm_ctx_t* ctx, const uint16_t* codebook, float* sqnorm, int64_t K, int64_t D,
                    ncm_stream_t stream) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if (K <= 0 || D <= 0 || D % 8 != 0 || !codebook || !sqnorm)
    return ncm_fail(NCM_EINVAL, "code_sqnorm: bad arguments (K=%lld D=%lld)", (long long)K, (long long)D);
  if (!aligned16(codebook)) return ncm_fail(NCM_EINVAL, "code_sqnorm: codebook must be 16-byte aligned");
  {
    Launch _launch(ctx, KID_SQNORM, static_cast<cudaStream_t>(stream));
    NCM_CUDA_TRY(launch_code_sqnorm(codebook, sqnorm, K, D, static_cast<cudaStream_t>(stream)));
  }
  return NCM_OK;
}

static int check_rvq_shape(int64_t N, int64_t D, int64_t K) {
  if (N <= 0 || D <= 0 || K <= 0 || N > INT32_MAX || K > INT32_MAX || D > 65536)
    return ncm_fail(NCM_EINVAL, "rvq: bad shape N=%lld D=%lld K=%lld", (long long)N, (long long)D, (long long)K);
  if (D % 8 != 0) return ncm_fail(NCM_EINVAL, "rvq: D=%lld must be a multiple of 8", (long long)D);
  return NCM_OK;
}

int ncm_rvq_level(ncm_ctx_t* ctx, float* residual, const uint16_t* codebook, const float* sqnorm, int32_t* codes,
                  int64_t N, int64_t D, int64_t K, ncm_stream_t stream) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if ((rc = check_rvq_shape(N, D, K))) return rc;
  if (!residual || !codebook || !codes) return ncm_fail(NCM_EINVAL, "rvq_level: null buffer");
  if (!aligned16(residual) || !aligned16(codebook) || !aligned16(codes) || (sqnorm && !aligned16(sqnorm)))
    return ncm_fail(NCM_EINVAL, "rvq_level: buffers must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const RvqPlan plan = rvq_plan(ctx->num_sms, N, K, true);
  WsCarver cv;
  const size_t o_sh = cv.take(2 * N * D);
  const size_t o_part = cv.take(plan.partial_bytes);
  const size_t o_sq = cv.take(sizeof(float) * K);
  uint8_t* ws = static_cast<uint8_t*>(ctx_workspace(ctx, cv.offset));
  if (ws == nullptr) return ncm_fail(NCM_ENOMEM, "rvq_level: workspace allocation failed");
  uint16_t* shadow = reinterpret_cast<uint16_t*>(ws + o_sh);
  if (sqnorm == nullptr) {
    float* sq = reinterpret_cast<float*>(ws + o_sq);
    {
      Launch _launch(ctx, KID_SQNORM, st);
      NCM_CUDA_TRY(launch_code_sqnorm(codebook, sq, K, D, st));
    }
    sqnorm = sq;
  }
  {
    Launch _launch(ctx, KID_CAST, st);
    NCM_CUDA_TRY(launch_f32_to_bf16(residual, shadow, N * D, st));
  }
  return rvq_level_core(ctx, shadow, nullptr, residual, nullptr, codebook, sqnorm, codes,
                        reinterpret_cast<RvqPartial*>(ws + o_part), plan, N, D, K, true, st);
}

int ncm_rvq_level_top2(ncm_ctx_t* ctx, float* residual, const uint16_t* codebook, const float* sqnorm,
                       int32_t* codes, float* top2_gap, int64_t N, int64_t D, int64_t K, ncm_stream_t stream) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if ((rc = check_rvq_shape(N, D, K))) return rc;
  if (!residual || !codebook || !codes || !top2_gap) return ncm_fail(NCM_EINVAL, "rvq_level_top2: null buffer");
  if (!aligned16(residual) || !aligned16(codebook) || !aligned16(codes) || (sqnorm && !aligned16(sqnorm)) ||
      (reinterpret_cast<uintptr_t>(top2_gap) & 3u))
    return ncm_fail(NCM_EINVAL, "rvq_level_top2: misaligned buffer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const RvqPlan plan = rvq_plan(ctx->num_sms, N, K);
  WsCarver cv;
  const size_t o_sh = cv.take(2 * N * D);
  const size_t o_part = cv.take(plan.partial_bytes);
  const size_t o_sq = cv.take(sizeof(float) * K);
  const size_t o_a2 = cv.take(sizeof(float) * N);
  const size_t o_d2 = cv.take(plan.splits > 1 ? sizeof(float) * plan.splits * N : 0);
  uint8_t* ws = static_cast<uint8_t*>(ctx_workspace(ctx, cv.offset));
  if (ws == nullptr) return ncm_fail(NCM_ENOMEM, "rvq_level_top2: workspace allocation failed");
  uint16_t* shadow = reinterpret_cast<uint16_t*>(ws + o_sh);
  if (sqnorm == nullptr) {
    float* sq = reinterpret_cast<float*>(ws + o_sq);
    {
      Launch _launch(ctx, KID_SQNORM, st);
      NCM_CUDA_TRY(launch_code_sqnorm(codebook, sq, K, D, st));
    }
    sqnorm = sq;
  }
  {
    Launch _launch(ctx, KID_CAST, st);
    NCM_CUDA_TRY(launch_f32_to_bf16(residual, shadow, N * D, st));
  }
  float* a2 = reinterpret_cast<float*>(ws + o_a2);
  {
    // ||bf16(r)||^2 per row: the same exact f64 sum of squares as the code norms
    Launch _launch(ctx, KID_SQNORM, st);
    NCM_CUDA_TRY(launch_code_sqnorm(shadow, a2, N, D, st));
  }
  RvqTop2 top2{top2_gap, a2, reinterpret_cast<float*>(ws + o_d2)};
  return rvq_level_core(ctx, shadow, nullptr, residual, nullptr, codebook, sqnorm, codes,
                        reinterpret_cast<RvqPartial*>(ws + o_part), plan, N, D, K, true, st, &top2);
}

int ncm_rvq_encode(ncm_ctx_t* ctx, const uint16_t* x, const uint16_t* codebooks, const float* sqnorms, int32_t L,
                   int32_t* codes, uint16_t* recon, float* residual_out, int64_t N, int64_t D, int64_t K,
                   ncm_stream_t stream) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if ((rc = check_rvq_shape(N, D, K))) return rc;
  if (L <= 0 || L > 64) return ncm_fail(NCM_EINVAL, "rvq_encode: L=%d must be in [1,64]", L);
  if (!x || !codebooks || !codes) return ncm_fail(NCM_EINVAL, "rvq_encode: null buffer");
  if (!aligned16(x) || !aligned16(codebooks) || !aligned16(codes) || (sqnorms && !aligned16(sqnorms)) ||
      (recon && !aligned16(recon)) || (residual_out && !aligned16(residual_out)))
    return ncm_fail(NCM_EINVAL, "rvq_encode: buffers must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const RvqPlan plan = rvq_plan(ctx->num_sms, N, K, true);
  WsCarver cv;
  const size_t o_sh = cv.take(2 * N * D);
  const size_t o_res = residual_out ? 0 : cv.take(sizeof(float) * N * D);
  const size_t o_part = cv.take(plan.partial_bytes);
  const size_t o_sq = sqnorms ? 0 : cv.take(sizeof(float) * K * L);
  uint8_t* ws = static_cast<uint8_t*>(ctx_workspace(ctx, cv.offset));
  if (ws == nullptr) return ncm_fail(NCM_ENOMEM, "rvq_encode: workspace allocation failed");
  if (sqnorms == nullptr) {
    float* sq = reinterpret_cast<float*>(ws + o_sq);
    {
      Launch _launch(ctx, KID_SQNORM, st);
      NCM_CUDA_TRY(launch_code_sqnorm(codebooks, sq, K * L, D, st));
    }
    sqnorms = sq;
  }
  return rvq_encode_core(ctx, x, codebooks, sqnorms, L, codes, recon,
                         residual_out ? residual_out : reinterpret_cast<float*>(ws + o_res), residual_out != nullptr,
                         reinterpret_cast<uint16_t*>(ws + o_sh), reinterpret_cast<RvqPartial*>(ws + o_part), plan, N,
                         D, K, st);
}

int ncm_rvq_encode_sharded(ncm_ctx_t* ctx, const uint16_t* x_local, const uint16_t* codebooks, const float* sqnorms,
                           int32_t L, int32_t* codes_all, uint16_t* recon_all, int64_t n_local, int64_t D, int64_t K,
                           ncm_stream_t stream) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if (ctx->comm == nullptr) return ncm_fail(NCM_EINVAL, "rvq_encode_sharded: no communicator (ncm_ctx_comm_init)");
  if ((rc = check_rvq_shape(n_local, D, K))) return rc;
  if (L <= 0 || L > 64) return ncm_fail(NCM_EINVAL, "rvq_encode_sharded: L=%d must be in [1,64]", L);
  if (!x_local || !codebooks || !codes_all) return ncm_fail(NCM_EINVAL, "rvq_encode_sharded: null buffer");
  if (!aligned16(x_local) || !aligned16(codebooks) || !aligned16(codes_all) || (sqnorms && !aligned16(sqnorms)) ||
      (recon_all && !aligned16(recon_all)))
    return ncm_fail(NCM_EINVAL, "rvq_encode_sharded: buffers must be 16-byte aligned");
  const int P = ctx->comm_size, me = ctx->comm_rank;
  const int64_t N = n_local * P;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const RvqPlan plan = rvq_plan(ctx->num_sms, n_local, K, true);
  WsCarver cv;
  const size_t o_sh = cv.take(2 * n_local * D);
  const size_t o_res = cv.take(sizeof(float) * n_local * D);
  const size_t o_part = cv.take(plan.partial_bytes);
  const size_t o_sq = sqnorms ? 0 : cv.take(sizeof(float) * K * L);
  const size_t o_codes = cv.take(sizeof(int32_t) * L * n_local);
  uint8_t* ws = static_cast<uint8_t*>(ctx_workspace(ctx, cv.offset));
  if (ws == nullptr) return ncm_fail(NCM_ENOMEM, "rvq_encode_sharded: workspace allocation failed");
  if (sqnorms == nullptr) {
    float* sq = reinterpret_cast<float*>(ws + o_sq);
    {
      Launch _launch(ctx, KID_SQNORM, st);
      NCM_CUDA_TRY(launch_code_sqnorm(codebooks, sq, K * L, D, st));
    }
    sqnorms = sq;
  }
  int32_t* codes_local = reinterpret_cast<int32_t*>(ws + o_codes);
  // this rank's reconstructions land in place, in its slice of recon_all
  uint16_t* recon_mine = recon_all ? recon_all + static_cast<size_t>(me) * n_local * D : nullptr;
  rc = rvq_encode_core(ctx, x_local, codebooks, sqnorms, L, codes_local, recon_mine,
                       reinterpret_cast<float*>(ws + o_res), false, reinterpret_cast<uint16_t*>(ws + o_sh),
                       reinterpret_cast<RvqPartial*>(ws + o_part), plan, n_local, D, K, st);
  if (rc) return rc;
  // codes [L, N]: one all-gather per level (rank r's rows sit at columns r*n..); recon [N, D] in place
  AllGatherItem items[65];
  int n = 0;
  for (int l = 0; l < L; ++l)
    items[n++] = AllGatherItem{codes_local + static_cast<size_t>(l) * n_local, codes_all + static_cast<size_t>(l) * N,
                               static_cast<size_t>(n_local), 4};
  if (recon_all) items[n++] = AllGatherItem{recon_mine, recon_all, static_cast<size_t>(n_local * D), 2};
  return comm_all_gather(ctx, items, n, st);
}

int ncm_rvq_encode_host(ncm_ctx_t* ctx, const uint16_t* x_host, const uint16_t* codebooks, const float* sqnorms,
                        int32_t L, int32_t* codes_host, uint16_t* recon_host, int64_t N, int64_t D, int64_t K,
                        ncm_stream_t stream) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if ((rc = check_rvq_shape(N, D, K))) return rc;
  if (L <= 0 || L > 64) return ncm_fail(NCM_EINVAL, "rvq_encode_host: L=%d must be in [1,64]", L);
  if (!x_host || !codebooks || !codes_host) return ncm_fail(NCM_EINVAL, "rvq_encode_host: null buffer");
  if (!aligned16(codebooks) || (sqnorms && !aligned16(sqnorms)))
    return ncm_fail(NCM_EINVAL, "rvq_encode_host: device buffers must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // Row chunks of about seven full waves of 128-row blocks (one wave = a
  // 128-row block per SM), so chunking adds no wave-quantisation loss; two
  // slots of device buffers alternate. A large encode starts and ends with a
  // two-wave chunk: the first copy in and the last copy out are the only
  // transfers nothing overlaps.
  const int64_t wave = static_cast<int64_t>(ctx->num_sms) * 128;
  std::vector<int64_t> starts;
  if (N >= 11 * wave) {
    const int64_t mid = (N - 4 * wave) / (7 * wave);
    starts.push_back(0);
    starts.push_back(2 * wave);
    for (int64_t i = 1; i <= mid; ++i) starts.push_back(2 * wave + i * 7 * wave);
    if (N - 2 * wave > starts.back()) starts.push_back(N - 2 * wave);  // the remainder, then the last two waves
  } else {
    const int64_t nchunks = std::max<int64_t>(1, std::min<int64_t>(16, (N + 7 * wave - 1) / (7 * wave)));
    const int64_t c0 = ((N + nchunks - 1) / nchunks + 127) / 128 * 128;
    for (int64_t r = 0; r < N; r += c0) starts.push_back(r);
  }
  starts.push_back(N);
  const int64_t nchunks = static_cast<int64_t>(starts.size()) - 1;
  int64_t C = 0;
  size_t part_bytes = 0;
  for (int64_t c = 0; c < nchunks; ++c) {
    const int64_t n = starts[c + 1] - starts[c];
    C = std::max(C, n);
    part_bytes = std::max(part_bytes, rvq_plan(ctx->num_sms, n, K, true).partial_bytes);
  }
  WsCarver cv;
  size_t o_x[2], o_codes[2], o_rec[2];
  for (int i = 0; i < 2; ++i) {
    o_x[i] = cv.take(2 * C * D);
    o_codes[i] = cv.take(sizeof(int32_t) * L * C);
    o_rec[i] = recon_host ? cv.take(2 * C * D) : 0;
  }
  const size_t o_res = cv.take(sizeof(float) * C * D);
  const size_t o_sh = cv.take(2 * C * D);
  const size_t o_part = cv.take(part_bytes);
  const size_t o_sq = sqnorms ? 0 : cv.take(sizeof(float) * K * L);
  uint8_t* ws = static_cast<uint8_t*>(ctx_workspace(ctx, cv.offset));
  if (ws == nullptr) return ncm_fail(NCM_ENOMEM, "rvq_encode_host: workspace allocation failed");
  if (ctx->copy_in == nullptr) {
    NCM_CUDA_TRY(cudaStreamCreateWithFlags(&ctx->copy_in, cudaStreamNonBlocking));
    NCM_CUDA_TRY(cudaStreamCreateWithFlags(&ctx->copy_out, cudaStreamNonBlocking));
    for (int i = 0; i < 2; ++i) {
      NCM_CUDA_TRY(cudaEventCreateWithFlags(&ctx->ev_in[i], cudaEventDisableTiming));
      NCM_CUDA_TRY(cudaEventCreateWithFlags(&ctx->ev_done[i], cudaEventDisableTiming));
      NCM_CUDA_TRY(cudaEventCreateWithFlags(&ctx->ev_out[i], cudaEventDisableTiming));
    }
  }
  if (sqnorms == nullptr) {
    float* sq = reinterpret_cast<float*>(ws + o_sq);
    Launch _launch(ctx, KID_SQNORM, st);
    NCM_CUDA_TRY(launch_code_sqnorm(codebooks, sq, K * L, D, st));
    sqnorms = sq;
  }
  float* resid = reinterpret_cast<float*>(ws + o_res);
  uint16_t* shadow = reinterpret_cast<uint16_t*>(ws + o_sh);
  RvqPartial* part = reinterpret_cast<RvqPartial*>(ws + o_part);
  for (int64_t c = 0; c < nchunks; ++c) {
    const int slot = static_cast<int>(c & 1);
    const int64_t r0 = starts[c];
    const int64_t n = starts[c + 1] - r0;
    if (n <= 0) break;
    uint16_t* xd = reinterpret_cast<uint16_t*>(ws + o_x[slot]);
    int32_t* cd = reinterpret_cast<int32_t*>(ws + o_codes[slot]);
    uint16_t* rd = recon_host ? reinterpret_cast<uint16_t*>(ws + o_rec[slot]) : nullptr;
    // rows in: the slot's previous chunk must be done computing
    if (c >= 2) NCM_CUDA_TRY(cudaStreamWaitEvent(ctx->copy_in, ctx->ev_done[slot], 0));
    NCM_CUDA_TRY(cudaMemcpyAsync(xd, x_host + r0 * D, 2 * n * D, cudaMemcpyHostToDevice, ctx->copy_in));
    NCM_CUDA_TRY(cudaEventRecord(ctx->ev_in[slot], ctx->copy_in));
    // compute: rows landed, and the slot's previous results are copied out
    NCM_CUDA_TRY(cudaStreamWaitEvent(st, ctx->ev_in[slot], 0));
    if (c >= 2) NCM_CUDA_TRY(cudaStreamWaitEvent(st, ctx->ev_out[slot], 0));
    const RvqPlan plan = rvq_plan(ctx->num_sms, n, K, true);
    if ((rc = rvq_encode_core(ctx, xd, codebooks, sqnorms, L, cd, rd, resid, false, shadow, part, plan, n, D, K, st)))
      return rc;
    NCM_CUDA_TRY(cudaEventRecord(ctx->ev_done[slot], st));
    // results out
    NCM_CUDA_TRY(cudaStreamWaitEvent(ctx->copy_out, ctx->ev_done[slot], 0));
    NCM_CUDA_TRY(cudaMemcpy2DAsync(codes_host + r0, sizeof(int32_t) * N, cd, sizeof(int32_t) * n,
                                   sizeof(int32_t) * n, L, cudaMemcpyDeviceToHost, ctx->copy_out));
    if (recon_host)
      NCM_CUDA_TRY(cudaMemcpyAsync(recon_host + r0 * D, rd, 2 * n * D, cudaMemcpyDeviceToHost, ctx->copy_out));
    NCM_CUDA_TRY(cudaEventRecord(ctx->ev_out[slot], ctx->copy_out));
  }
  NCM_CUDA_TRY(cudaStreamSynchronize(ctx->copy_out));
  return ncm_sync(ctx, stream);
}

int ncm_pool_avg(ncm_ctx_t* ctx, const float* x, float* y, int64_t B, int64_t T, int64_t D, int32_t factor,
                 ncm_stream_t stream) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if (B <= 0 || T <= 0 || D <= 0 || factor <= 0 || T % factor != 0 || D % 4 != 0 || !x || !y)
    return ncm_fail(NCM_EINVAL, "pool_avg: bad arguments (B=%lld T=%lld D=%lld factor=%d)", (long long)B,
                    (long long)T, (long long)D, factor);
  if (!aligned16(x) || !aligned16(y)) return ncm_fail(NCM_EINVAL, "pool_avg: buffers must be 16-byte aligned");
  {
    Launch _launch(ctx, KID_POOL, static_cast<cudaStream_t>(stream));
    NCM_CUDA_TRY(launch_pool_avg(x, y, nullptr, B, T, D, factor, static_cast<cudaStream_t>(stream)));
  }
  return NCM_OK;
}

int ncm_rvq_decode(ncm_ctx_t* ctx, const int32_t* codes, const uint16_t* codebooks, int32_t L, uint16_t* recon,
                   int64_t N, int64_t D, int64_t K, ncm_stream_t stream) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if ((rc = check_rvq_shape(N, D, K))) return rc;
  if (L <= 0 || !codes || !codebooks || !recon) return ncm_fail(NCM_EINVAL, "rvq_decode: bad arguments");
  if (!aligned16(codes) || !aligned16(codebooks) || !aligned16(recon))
    return ncm_fail(NCM_EINVAL, "rvq_decode: buffers must be 16-byte aligned");
  {
    Launch _launch(ctx, KID_DECODE, static_cast<cudaStream_t>(stream));
    NCM_CUDA_TRY(launch_rvq_decode(codes, codebooks, L, recon, nullptr, N, D, K, ctx->d_err,
                                 static_cast<cudaStream_t>(stream)));
  }
  return NCM_OK;
}

}  // extern "C"

namespace {

// Shape checks shared by the tokenizer and the multiscale decode.
int check_tokenizer_cfg(const ncm_tokenizer_config_t* cfg, bool with_projections, const uint16_t* phi_weight,
                        const float* phi_bias) {
  if (cfg == nullptr) return ncm_fail(NCM_EINVAL, "tokenizer: null config");
  const int64_t B = cfg->batch, T = cfg->seq_len, Din = cfg->model_width;
  const int S = cfg->num_scales, L = cfg->levels_per_scale;
  if (B <= 0 || T <= 0 || S <= 0 || S > 16 || L <= 0 || L > 64 || (with_projections && (Din <= 0 || Din % 8 != 0)))
    return ncm_fail(NCM_EINVAL, "tokenizer: bad config");
  int rc = check_rvq_shape(B * T, cfg->vq_width, cfg->codebook_size);
  if (rc) return rc;
  for (int s = 0; s < S; ++s)
    if (cfg->pool_factors[s] <= 0 || T % cfg->pool_factors[s] != 0)
      return ncm_fail(NCM_EINVAL, "tokenizer: pool factor %d does not divide T=%lld", cfg->pool_factors[s],
                      (long long)T);
  if (cfg->upsample_mode != 0 && cfg->upsample_mode != 1)
    return ncm_fail(NCM_EINVAL, "tokenizer: upsample_mode %d unknown", cfg->upsample_mode);
  if ((phi_weight == nullptr) != (phi_bias == nullptr))
    return ncm_fail(NCM_EINVAL, "tokenizer: pass both Phi weight and bias, or neither");
  if (phi_weight != nullptr) {
    if (!(cfg->phi_ratio >= 0.f && cfg->phi_ratio <= 1.f))
      return ncm_fail(NCM_EINVAL, "tokenizer: phi_ratio must lie in [0, 1]");
    if (B * (T + 1) + 1 > INT32_MAX / 2) return ncm_fail(NCM_EINVAL, "tokenizer: too many rows for Phi");
    if ((reinterpret_cast<uintptr_t>(phi_weight) & 1u) || !aligned16(phi_bias))
      return ncm_fail(NCM_EINVAL, "tokenizer: Phi buffers misaligned (bias must be 16-byte aligned)");
  }
  return NCM_OK;
}

// Workspace of the general per-scale step (linear upsampling and/or Phi).
struct ScaleEmitWs {
  float* acc = nullptr;        // [N, D] f32 reconstruction accumulator
  float* qf = nullptr;         // [N, D] f32 upsampled q (Phi's blend input)
  uint16_t* qpad = nullptr;    // padded bf16 copy of qf (Phi's GEMM operand)
  uint16_t* w_pack = nullptr;  // [S, D, 3 * dp] tap-major Phi kernels
  int64_t dp = 0;
};

// Q = up(q_s); with Phi Q = (1 - r) Q + r (bias + conv(Q)); resid -= Q (if
// given); acc += Q.
int scale_emit(ncm_ctx* ctx, const ncm_tokenizer_config_t* cfg, int s, const float* q, float* resid,
               const ScaleEmitWs& w, const float* phi_bias, cudaStream_t st) {
  const int64_t B = cfg->batch, T = cfg->seq_len, D = cfg->vq_width;
  const int64_t Tq = T / cfg->pool_factors[s];
  if (w.w_pack == nullptr) {
    Launch _launch(ctx, KID_UPSAMPLE, st);
    NCM_CUDA_TRY(launch_upsample(q, B, Tq, T, D, cfg->upsample_mode, nullptr, nullptr, 0, resid, w.acc, st));
    return NCM_OK;
  }
  {
    Launch _launch(ctx, KID_UPSAMPLE, st);
    NCM_CUDA_TRY(launch_upsample(q, B, Tq, T, D, cfg->upsample_mode, w.qf, w.qpad, w.dp, nullptr, nullptr, st));
  }
  SegMap map{};
  map.seg_len = static_cast<int>(T);
  map.nseg = static_cast<int>(B);
  ConvEpilogue ep{};
  ep.x_f32 = w.qf;
  ep.resid = resid;
  ep.acc_f32 = w.acc;
  ep.bias = phi_bias + s * D;
  ep.alpha = 1.f - cfg->phi_ratio;
  ep.beta = cfg->phi_ratio;
  return conv3_gemm(ctx, w.qpad, w.w_pack + static_cast<size_t>(s) * D * 3 * w.dp, map, w.dp, D, ep, st);
}

// Carves the general step's buffers (nothing when nearest and no Phi).
struct ScaleEmitCarve {
  size_t o_acc = 0, o_qf = 0, o_qpad = 0, o_w = 0;
  bool general = false, phi = false;
};
ScaleEmitCarve carve_scale_emit(WsCarver& cv, const ncm_tokenizer_config_t* cfg, bool phi) {
  ScaleEmitCarve c;
  c.general = cfg->upsample_mode != 0 || phi;
  c.phi = phi;
  if (!c.general) return c;
  const int64_t N = cfg->batch * cfg->seq_len, D = cfg->vq_width, dp = (D + 63) / 64 * 64;
  c.o_acc = cv.take(sizeof(float) * N * D);
  if (phi) {
    c.o_qf = cv.take(sizeof(float) * N * D);
    c.o_qpad = cv.take(2 * (cfg->batch * (cfg->seq_len + 1) + 1) * dp);
    c.o_w = cv.take(2 * static_cast<size_t>(cfg->num_scales) * D * 3 * dp);
  }
  return c;
}
int setup_scale_emit(ncm_ctx* ctx, const ScaleEmitCarve& c, uint8_t* ws, const ncm_tokenizer_config_t* cfg,
                     const uint16_t* phi_weight, ScaleEmitWs* w, cudaStream_t st) {
  if (!c.general) return NCM_OK;
  const int64_t N = cfg->batch * cfg->seq_len, D = cfg->vq_width;
  w->dp = (D + 63) / 64 * 64;
  w->acc = reinterpret_cast<float*>(ws + c.o_acc);
  NCM_CUDA_TRY(cudaMemsetAsync(w->acc, 0, sizeof(float) * N * D, st));
  if (!c.phi) return NCM_OK;
  w->qf = reinterpret_cast<float*>(ws + c.o_qf);
  w->qpad = reinterpret_cast<uint16_t*>(ws + c.o_qpad);
  w->w_pack = reinterpret_cast<uint16_t*>(ws + c.o_w);
  for (int s = 0; s < cfg->num_scales; ++s) {
    Launch _launch(ctx, KID_CAST, st);
    NCM_CUDA_TRY(launch_conv_repack(phi_weight + static_cast<size_t>(s) * D * D * 3, nullptr,
                                    w->w_pack + static_cast<size_t>(s) * D * 3 * w->dp, D, w->dp, st));
  }
  return NCM_OK;
}

}  // namespace

extern "C" {

int ncm_tokenizer_forward(ncm_ctx_t* ctx, const ncm_tokenizer_config_t* cfg, const uint16_t* x, const uint16_t* w_in,
                          const uint16_t* b_in, const uint16_t* codebooks, const float* sqnorms,
                          const uint16_t* w_out, const uint16_t* b_out, int32_t* codes, uint16_t* recon, uint16_t* y,
                          ncm_stream_t stream) {
  return ncm_tokenizer_forward_ex(ctx, cfg, x, w_in, b_in, codebooks, sqnorms, nullptr, nullptr, w_out, b_out, codes,
                                  recon, y, stream);
}

int ncm_tokenizer_forward_ex(ncm_ctx_t* ctx, const ncm_tokenizer_config_t* cfg, const uint16_t* x,
                             const uint16_t* w_in, const uint16_t* b_in, const uint16_t* codebooks,
                             const float* sqnorms, const uint16_t* phi_weight, const float* phi_bias,
                             const uint16_t* w_out, const uint16_t* b_out, int32_t* codes, uint16_t* recon,
                             uint16_t* y, ncm_stream_t stream) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if ((rc = check_tokenizer_cfg(cfg, true, phi_weight, phi_bias))) return rc;
  const int64_t B = cfg->batch, T = cfg->seq_len, Din = cfg->model_width, D = cfg->vq_width, K = cfg->codebook_size;
  const int S = cfg->num_scales, L = cfg->levels_per_scale;
  if (!x || !w_in || !codebooks || !w_out || !codes || !y)
    return ncm_fail(NCM_EINVAL, "tokenizer: null buffer");
  if (!aligned16(x) || !aligned16(w_in) || !aligned16(codebooks) || !aligned16(w_out) || !aligned16(codes) ||
      !aligned16(y) || (recon && !aligned16(recon)) || (sqnorms && !aligned16(sqnorms)) ||
      (b_in && !aligned16(b_in)) || (b_out && !aligned16(b_out)))
    return ncm_fail(NCM_EINVAL, "tokenizer: buffers must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t N = B * T;
  int64_t max_rows = 0;
  for (int s = 0; s < S; ++s) max_rows = std::max<int64_t>(max_rows, N / cfg->pool_factors[s]);
  size_t part_bytes = 0;
  for (int s = 0; s < S; ++s)
    part_bytes = std::max(part_bytes, rvq_plan(ctx->num_sms, N / cfg->pool_factors[s], K, true).partial_bytes);
  WsCarver cv;
  const size_t o_h = cv.take(2 * N * D);
  const size_t o_r = cv.take(sizeof(float) * N * D);
  size_t o_q[16];
  for (int s = 0; s < S; ++s) o_q[s] = cv.take(sizeof(float) * (N / cfg->pool_factors[s]) * D);
  const size_t o_u = cv.take(sizeof(float) * max_rows * D);
  const size_t o_ub = cv.take(2 * max_rows * D);
  const size_t o_rb = recon ? 0 : cv.take(2 * N * D);
  const size_t o_part = cv.take(part_bytes);
  const size_t o_sq = sqnorms ? 0 : cv.take(sizeof(float) * S * L * K);
  const ScaleEmitCarve ec = carve_scale_emit(cv, cfg, phi_weight != nullptr);
  uint8_t* ws = static_cast<uint8_t*>(ctx_workspace(ctx, cv.offset));
  if (ws == nullptr) return ncm_fail(NCM_ENOMEM, "tokenizer: workspace allocation failed");
  uint16_t* h = reinterpret_cast<uint16_t*>(ws + o_h);
  float* r = reinterpret_cast<float*>(ws + o_r);
  float* q[16];
  for (int s = 0; s < S; ++s) q[s] = reinterpret_cast<float*>(ws + o_q[s]);
  float* u = reinterpret_cast<float*>(ws + o_u);
  uint16_t* ub = reinterpret_cast<uint16_t*>(ws + o_ub);
  uint16_t* rb = recon ? recon : reinterpret_cast<uint16_t*>(ws + o_rb);
  RvqPartial* part = reinterpret_cast<RvqPartial*>(ws + o_part);
  ScaleEmitWs ew;
  if ((rc = setup_scale_emit(ctx, ec, ws, cfg, phi_weight, &ew, st))) return rc;
  if (sqnorms == nullptr) {
    float* sq = reinterpret_cast<float*>(ws + o_sq);
    {
      Launch _launch(ctx, KID_SQNORM, st);
      NCM_CUDA_TRY(launch_code_sqnorm(codebooks, sq, static_cast<int64_t>(S) * L * K, D, st));
    }
    sqnorms = sq;
  }
  // input projection, then the f32 residual and the first scale's pooled rows
  rc = linear_bf16(ctx, x, w_in, b_in, h, nullptr, N, Din, D, st);
  if (rc) return rc;
  {
    Launch _launch(ctx, KID_CAST, st);
    NCM_CUDA_TRY(launch_bf16_to_f32(h, r, N * D, st));
  }
  {
    Launch _launch(ctx, KID_POOL, st);
    NCM_CUDA_TRY(launch_pool_avg(r, u, ub, B, T, D, cfg->pool_factors[0], st));
  }
  int32_t* codes_s = codes;
  for (int s = 0; s < S; ++s) {
    const int f = cfg->pool_factors[s];
    const int64_t rows = N / f;
    const RvqPlan plan = rvq_plan(ctx->num_sms, rows, K, true);
    for (int l = 0; l < L; ++l) {
      const size_t cb_off = (static_cast<size_t>(s) * L + l) * K;
      rc = rvq_level_core(ctx, ub, nullptr, u, l == L - 1 ? nullptr : ub, codebooks + cb_off * D, sqnorms + cb_off,
                          codes_s + static_cast<size_t>(l) * rows, part, plan, rows, D, K, l != L - 1, st);
      if (rc) return rc;
    }
    const bool next = s + 1 < S;
    const int g = next ? cfg->pool_factors[s + 1] : 0;
    const uint16_t* cbs_s = codebooks + static_cast<size_t>(s) * L * K * D;
    if (!ec.general) {
      // q_s, and r -= up(q_s) with the next scale's pooling in the same pass
      const bool fused_pool = next && f % g == 0;
      {
        Launch _launch(ctx, KID_SCALE_UPDATE, st);
        NCM_CUDA_TRY(launch_scale_advance(codes_s, cbs_s, L, r, q[s], u, ub, rows, D, K, f, fused_pool ? g : 0, next,
                                          ctx->d_err, st));
      }
      if (next && !fused_pool) {
        Launch _launch(ctx, KID_POOL, st);
        NCM_CUDA_TRY(launch_pool_avg(r, u, ub, B, T, D, g, st));
      }
    } else {
      {
        Launch _launch(ctx, KID_SCALE_UPDATE, st);
        NCM_CUDA_TRY(launch_scale_advance(codes_s, cbs_s, L, nullptr, q[s], nullptr, nullptr, rows, D, K, f, 0, false,
                                          ctx->d_err, st));
      }
      if ((rc = scale_emit(ctx, cfg, s, q[s], next ? r : nullptr, ew, phi_bias, st))) return rc;
      if (next) {
        Launch _launch(ctx, KID_POOL, st);
        NCM_CUDA_TRY(launch_pool_avg(r, u, ub, B, T, D, g, st));
      }
    }
    codes_s += static_cast<size_t>(L) * rows;
  }
  {
    // recon = bf16(sum_s Q_s), scales in order
    Launch _launch(ctx, KID_CAST, st);
    if (ec.general)
      NCM_CUDA_TRY(launch_f32_to_bf16(ew.acc, rb, N * D, st));
    else
      NCM_CUDA_TRY(launch_multiscale_recon(q, cfg->pool_factors, S, rb, N, D, st));
  }
  return linear_bf16(ctx, rb, w_out, b_out, y, nullptr, N, D, Din, st);
}

int ncm_multiscale_decode(ncm_ctx_t* ctx, const ncm_tokenizer_config_t* cfg, const int32_t* codes,
                          const uint16_t* codebooks, const uint16_t* phi_weight, const float* phi_bias,
                          uint16_t* recon, ncm_stream_t stream) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if ((rc = check_tokenizer_cfg(cfg, false, phi_weight, phi_bias))) return rc;
  if (!codes || !codebooks || !recon) return ncm_fail(NCM_EINVAL, "multiscale_decode: null buffer");
  if (!aligned16(codes) || !aligned16(codebooks) || !aligned16(recon))
    return ncm_fail(NCM_EINVAL, "multiscale_decode: buffers must be 16-byte aligned");
  const int64_t N = cfg->batch * cfg->seq_len, D = cfg->vq_width, K = cfg->codebook_size;
  const int S = cfg->num_scales, L = cfg->levels_per_scale;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  WsCarver cv;
  size_t o_q[16];
  for (int s = 0; s < S; ++s) o_q[s] = cv.take(sizeof(float) * (N / cfg->pool_factors[s]) * D);
  const ScaleEmitCarve ec = carve_scale_emit(cv, cfg, phi_weight != nullptr);
  uint8_t* ws = static_cast<uint8_t*>(ctx_workspace(ctx, cv.offset));
  if (ws == nullptr) return ncm_fail(NCM_ENOMEM, "multiscale_decode: workspace allocation failed");
  float* q[16];
  for (int s = 0; s < S; ++s) q[s] = reinterpret_cast<float*>(ws + o_q[s]);
  ScaleEmitWs ew;
  if ((rc = setup_scale_emit(ctx, ec, ws, cfg, phi_weight, &ew, st))) return rc;
  const int32_t* codes_s = codes;
  for (int s = 0; s < S; ++s) {
    const int64_t rows = N / cfg->pool_factors[s];
    {
      Launch _launch(ctx, KID_SCALE_UPDATE, st);
      NCM_CUDA_TRY(launch_scale_advance(codes_s, codebooks + static_cast<size_t>(s) * L * K * D, L, nullptr, q[s],
                                        nullptr, nullptr, rows, D, K, cfg->pool_factors[s], 0, false, ctx->d_err, st));
    }
    if (ec.general && (rc = scale_emit(ctx, cfg, s, q[s], nullptr, ew, phi_bias, st))) return rc;
    codes_s += static_cast<size_t>(L) * rows;
  }
  Launch _launch(ctx, KID_CAST, st);
  if (ec.general)
    NCM_CUDA_TRY(launch_f32_to_bf16(ew.acc, recon, N * D, st));
  else
    NCM_CUDA_TRY(launch_multiscale_recon(q, cfg->pool_factors, S, recon, N, D, st));
  return NCM_OK;
}

int ncm_profile_enable(ncm_ctx_t* ctx, int on) {
  if (ctx == nullptr) return ncm_fail(NCM_EINVAL, "null context");
  ctx->prof.on = on != 0;
  return NCM_OK;
}

int ncm_profile_read(ncm_ctx_t* ctx, const char* kernel, double* total_ms, int64_t* launches) {
  int rc = check_ctx(ctx);
  if (rc) return rc;
  if (kernel == nullptr) return ncm_fail(NCM_EINVAL, "profile_read: null kernel name");
  const bool all = std::strcmp(kernel, "*") == 0;
  int which = -1;
  for (int i = 0; i < KID_COUNT; ++i)
    if (std::strcmp(kernel, kKernelNames[i]) == 0) which = i;
  if (!all && which < 0) return ncm_fail(NCM_EINVAL, "profile_read: unknown kernel family '%s'", kernel);
  double ms = 0.0;
  long long n = 0;
  for (int i = 0; i < KID_COUNT; ++i) {
    if (!all && i != which) continue;
    ProfState& p = ctx->prof;
    for (size_t j = 0; j < p.used[i]; ++j) {
      NCM_CUDA_TRY(cudaEventSynchronize(p.events[i][j].second));
      float e = 0.f;
      NCM_CUDA_TRY(cudaEventElapsedTime(&e, p.events[i][j].first, p.events[i][j].second));
      ms += e;
    }
    n += p.launches[i];
    p.used[i] = 0;
    p.launches[i] = 0;
  }
  if (total_ms) *total_ms = ms;
  if (launches) *launches = n;
  return NCM_OK;
}

}  // extern "C"
