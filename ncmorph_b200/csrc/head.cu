// Codebook-tied output head of the NCM generator (_TiedCodebookHead,
// PROJECT.md:222; decision D18 at PROJECT.md:471):
//     E_sq[k]  = sum_d E[k,d]^2            d_scale = mean_k E_sq[k]
//     logits   = (2 z.E^T - E_sq) / d_scale * exp(log_inv_T) + bias
// It is the RVQ distance GEMM with another epilogue. With s = exp(log_inv_T)
// / d_scale and per-code offsets c_k = s E_sq[k] - bias[k], logits =
// fmaf(2 s, z.E_k, -c_k) (one FMA per logit; the module's own order, with a
// division per element, differs from it by rounding only). Two forms:
//   * ncm_tied_head_logits writes the [T, K] logits (tcgen05 GEMM, mode-4
//     epilogue in gemm.cu);
//   * ncm_tied_head_argmax returns argmax_k logits (the temperature-0 pick of
//     _sample_level_raw) without materialising them: -logits =
//     fmaf(-2 s, z.E_k, c_k), so the RVQ argmin kernel runs with multiplier
//     -2 s and the offsets c_k.
#include <algorithm>

#include "internal.h"

namespace ncm {
namespace {

// One block: d_scale = f32(sum_k f64(E_sq[k]) / K), e = exp(log_inv_T),
// s = e / d_scale; scal = {d_scale, e, -2 s}; c[k] = s E_sq[k] - bias[k].
__global__ void __launch_bounds__(1024) head_prep_kernel(const float* __restrict__ esq,
                                                         const float* __restrict__ bias, int K, float log_inv_T,
                                                         float* __restrict__ scal, float* __restrict__ c) {
  __shared__ double part[32];
  __shared__ float s_sh;
  double acc = 0.0;
  for (int k = threadIdx.x; k < K; k += blockDim.x) acc += static_cast<double>(esq[k]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < (static_cast<int>(blockDim.x) + 31) / 32; ++w) t += part[w];
    const float dsc = static_cast<float>(t / K);
    const float e = expf(log_inv_T);
    const float sc = __fdiv_rn(e, dsc);
    scal[0] = dsc;
    scal[1] = e;
    scal[2] = -2.f * sc;
    s_sh = sc;
  }
  __syncthreads();
  if (c == nullptr) return;
  const float sc = s_sh;
  for (int k = threadIdx.x; k < K; k += blockDim.x)
    c[k] = __fsub_rn(__fmul_rn(sc, esq[k]), bias != nullptr ? bias[k] : 0.f);
}

bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int head_ctx_ok(ncm_ctx* ctx) {
  if (ctx == nullptr) return ncm_fail(NCM_EINVAL, "null context");
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev != ctx->device) {
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e != cudaSuccess) return ncm_set_cuda_error(e);
  }
  return NCM_OK;
}

int check_head(const uint16_t* z, const uint16_t* codebook, const float* esq, const float* bias, int64_t T,
               int64_t d, int64_t K) {
  if (T <= 0 || d <= 0 || K <= 0 || T > INT32_MAX || K > INT32_MAX || d > INT32_MAX)
    return ncm_fail(NCM_EINVAL, "tied head: bad shape T=%lld d=%lld K=%lld", (long long)T, (long long)d,
                    (long long)K);
  if (d % 8 != 0) return ncm_fail(NCM_EINVAL, "tied head: d=%lld must be a multiple of 8", (long long)d);
  if (!z || !codebook) return ncm_fail(NCM_EINVAL, "tied head: null buffer");
  if (!a16(z) || !a16(codebook) || !a16(esq) || !a16(bias))
    return ncm_fail(NCM_EINVAL, "tied head: buffers must be 16-byte aligned");
  return NCM_OK;
}

}  // namespace
}  // namespace ncm

using namespace ncm;

extern "C" {

int ncm_tied_head_logits(ncm_ctx_t* ctx, const uint16_t* z, const uint16_t* codebook, const float* esq,
                         const float* bias, float log_inv_T, float* logits, int64_t T, int64_t d, int64_t K,
                         ncm_stream_t stream) {
  int rc = head_ctx_ok(ctx);
  if (rc) return rc;
  if ((rc = check_head(z, codebook, esq, bias, T, d, K))) return rc;
  if (!logits || !a16(logits)) return ncm_fail(NCM_EINVAL, "tied head: logits must be a 16-byte aligned buffer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  WsCarver cv;
  const size_t o_sq = cv.take(esq ? 0 : sizeof(float) * K);
  const size_t o_sc = cv.take(4 * sizeof(float));
  const size_t o_c = cv.take(sizeof(float) * K);
  uint8_t* ws = static_cast<uint8_t*>(ctx_workspace(ctx, cv.offset));
  if (ws == nullptr) return ncm_fail(NCM_ENOMEM, "tied head: workspace allocation failed");
  float* scal = reinterpret_cast<float*>(ws + o_sc);
  float* c = reinterpret_cast<float*>(ws + o_c);
  if (esq == nullptr) {
    float* sq = reinterpret_cast<float*>(ws + o_sq);
    Launch _launch(ctx, KID_SQNORM, st);
    NCM_CUDA_TRY(launch_code_sqnorm(codebook, sq, K, d, st));
    esq = sq;
  }
  {
    Launch _launch(ctx, KID_CAST, st);
    head_prep_kernel<<<1, 1024, 0, st>>>(esq, bias, static_cast<int>(K), log_inv_T, scal, c);
    NCM_CUDA_TRY(cudaGetLastError());
  }
  return tied_head_logits_gemm(ctx, z, codebook, c, scal, logits, T, d, K, st);
}

int ncm_tied_head_argmax(ncm_ctx_t* ctx, const uint16_t* z, const uint16_t* codebook, const float* esq,
                         const float* bias, float log_inv_T, int32_t* codes, int64_t T, int64_t d, int64_t K,
                         ncm_stream_t stream) {
  int rc = head_ctx_ok(ctx);
  if (rc) return rc;
  if ((rc = check_head(z, codebook, esq, bias, T, d, K))) return rc;
  if (!codes || !a16(codes)) return ncm_fail(NCM_EINVAL, "tied head: codes must be a 16-byte aligned buffer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const RvqPlan plan = rvq_plan(ctx->num_sms, T, K);
  WsCarver cv;
  const size_t o_sq = cv.take(esq ? 0 : sizeof(float) * K);
  const size_t o_sc = cv.take(4 * sizeof(float));
  const size_t o_c = cv.take(sizeof(float) * K);
  const size_t o_part = cv.take(plan.partial_bytes);
  uint8_t* ws = static_cast<uint8_t*>(ctx_workspace(ctx, cv.offset));
  if (ws == nullptr) return ncm_fail(NCM_ENOMEM, "tied head: workspace allocation failed");
  float* scal = reinterpret_cast<float*>(ws + o_sc);
  float* c = reinterpret_cast<float*>(ws + o_c);
  RvqPartial* part = reinterpret_cast<RvqPartial*>(ws + o_part);
  if (esq == nullptr) {
    float* sq = reinterpret_cast<float*>(ws + o_sq);
    Launch _launch(ctx, KID_SQNORM, st);
    NCM_CUDA_TRY(launch_code_sqnorm(codebook, sq, K, d, st));
    esq = sq;
  }
  {
    Launch _launch(ctx, KID_CAST, st);
    head_prep_kernel<<<1, 1024, 0, st>>>(esq, bias, static_cast<int>(K), log_inv_T, scal, c);
    NCM_CUDA_TRY(cudaGetLastError());
  }
  CUtensorMap tmA, tmB;
  if (!make_tmap_bf16_2d(&tmA, z, T, d, 128) || !make_tmap_bf16_2d(&tmB, codebook, K, d, 256))
    return ncm_fail(NCM_EINVAL, "tied head: tensor map encoding failed (T=%lld d=%lld K=%lld)", (long long)T,
                    (long long)d, (long long)K);
  int* counters = plan.splits > 1 ? rvq_counters(ctx, plan.row_blocks) : nullptr;
  {
    Launch _launch(ctx, KID_RVQ_ARGMIN, st);
    NCM_CUDA_TRY(launch_rvq_argmin(plan, tmA, tmB, c, codes, part, ctx->d_err, T, d, K, st, nullptr, nullptr,
                                   scal + 2, counters));
  }
  if (plan.splits > 1 && counters == nullptr) {
    Launch _launch(ctx, KID_RVQ_APPLY, st);
    NCM_CUDA_TRY(launch_rvq_apply(plan, part, codes, nullptr, nullptr, nullptr, codebook, ctx->d_err, T, d, K, false,
                                  st));
  }
  return NCM_OK;
}

}  // extern "C"
