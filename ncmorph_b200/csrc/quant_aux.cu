// The quantiser's remaining pieces around the RVQ levels
// (research/reference/vq_forward_semantics.md):
//
//  * pre-quantisation GroupNorm, affine=False (:43-49; upstream
//    models/vqvae.py:66, :82, :86): per sample and group, statistics over all
//    positions and the group's channels (f64 sums), y = (x - mean) * rstd;
//  * the learned level-0 cascade (:127-139): Conv1d(C, C, kernel 4,
//    stride 4) down and ConvTranspose1d(C, C, kernel 4, stride 4) up. On
//    [B, L, C] rows both are GEMMs on the tcgen05 linear kernel: four
//    consecutive rows are one contiguous row of 4C values, so
//      down: y[B*L/4, C]  = x viewed as [B*L/4, 4C] . Wd^T (+ b),
//            Wd[o][t*C + i] = w[o][i][t]   (Conv1d weight [C_out, C_in, 4])
//      up:   y[B*L, 4C]   = x[B*L, C] . Wu^T (+ b tiled 4x), viewed as [B*4L, C],
//            Wu[t*C + o][i] = w[i][o][t]   (ConvTranspose1d weight [C_in, C_out, 4]);
//  * the codebook EMA (:141-173; models/quant.py:485-500): per code the count
//    and the sum of the rows assigned to it, then N <- g N + (1-g) n,
//    m <- g m + (1-g) s, Laplace-smoothed counts and e = m / N_hat. Rows are
//    grouped by code with a counting sort (a stable scatter by row index), so
//    each code's sum runs over its rows in increasing row order: the result is
//    the same on every run (no floating-point atomics).
#include <algorithm>
#include <cmath>

#include "internal.h"
#include "ptx.cuh"

namespace ncm {
namespace {

int blocks_of(long long n, int per) { return static_cast<int>((n + per - 1) / per); }

// ------------------------------------------------------------- GroupNorm
// Three passes so every SM takes part: (1) block (sample*group, chunk) sums a
// slab of rows of one group in f64 into partials[sg][chunk]; (2) one thread
// per (sample, group) adds its partials in chunk order (the same bits every
// run) into mean and 1/sqrt(var + eps); (3) an elementwise pass normalises
// four channels per thread.
constexpr int kGnChunks = 32;

// VEC: the group's channels are read as float4 (C / G a multiple of 4, x 16-byte aligned)
template <bool VEC>
__global__ void __launch_bounds__(256) group_norm_partial_kernel(const float* __restrict__ x, int T, int C, int G,
                                                                 double2* __restrict__ part) {
  const int sg = blockIdx.x;
  const int b = sg / G, g = sg - (sg / G) * G;
  constexpr int W = VEC ? 4 : 1;
  const unsigned cw = static_cast<unsigned>(C / G / W);  // vectors per row of the group
  const int t0 = static_cast<int>((static_cast<long long>(T) * blockIdx.y) / kGnChunks);
  const int t1 = static_cast<int>((static_cast<long long>(T) * (blockIdx.y + 1)) / kGnChunks);
  const float* xb = x + static_cast<size_t>(b) * T * C + static_cast<size_t>(g) * (C / G);
  // rows of a chunk x vectors of a row stay below 2^32 for any T, C below 2^31 split 32 ways
  const unsigned n = static_cast<unsigned>(t1 - t0) * cw;
  double s = 0.0, ss = 0.0;
  for (unsigned i = threadIdx.x; i < n; i += blockDim.x) {
    const unsigned r = i / cw;
    const float* px = xb + static_cast<size_t>(t0 + r) * C + (i - r * cw) * W;
    if constexpr (VEC) {
      const float4 v = *reinterpret_cast<const float4*>(px);
      s += static_cast<double>(v.x) + static_cast<double>(v.y) + static_cast<double>(v.z) + static_cast<double>(v.w);
      ss = __fma_rn(static_cast<double>(v.x), v.x, ss);
      ss = __fma_rn(static_cast<double>(v.y), v.y, ss);
      ss = __fma_rn(static_cast<double>(v.z), v.z, ss);
      ss = __fma_rn(static_cast<double>(v.w), v.w, ss);
    } else {
      const float v = *px;
      s += v;
      ss = __fma_rn(static_cast<double>(v), v, ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, o);
    ss += __shfl_xor_sync(0xffffffffu, ss, o);
  }
  __shared__ double red[2][8];
  if ((threadIdx.x & 31) == 0) red[0][threadIdx.x >> 5] = s, red[1][threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    double a = 0.0, q = 0.0;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) a += red[0][w], q += red[1][w];
    part[static_cast<size_t>(sg) * kGnChunks + blockIdx.y] = make_double2(a, q);
  }
}

__global__ void __launch_bounds__(256) group_norm_stats_kernel(const double2* __restrict__ part, int n_sg,
                                                               long long count, float eps, float2* __restrict__ stat) {
  const int sg = blockIdx.x * blockDim.x + threadIdx.x;
  if (sg >= n_sg) return;
  double a = 0.0, q = 0.0;
  for (int c = 0; c < kGnChunks; ++c) {
    const double2 v = part[static_cast<size_t>(sg) * kGnChunks + c];
    a += v.x;
    q += v.y;
  }
  const double mean = a / count;
  const double var = fmax(q / count - mean * mean, 0.0);  // biased variance, as GroupNorm
  stat[sg] = make_float2(static_cast<float>(mean), static_cast<float>(1.0 / sqrt(var + eps)));
}

// VEC: four elements per thread (C / G a multiple of 4, 16-byte aligned
// buffers: the four share a group); otherwise one element per thread
template <bool VEC>
__global__ void __launch_bounds__(256) group_norm_apply_kernel(const float* __restrict__ x, float* __restrict__ y,
                                                               long long n, int T, int C, int G,
                                                               const float2* __restrict__ stat) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  constexpr int W = VEC ? 4 : 1;
  if (i * W >= n) return;
  const long long e = i * W;
  const int c = static_cast<int>(e % C);
  const long long b = e / (static_cast<long long>(T) * C);
  const float2 st = stat[b * G + c / (C / G)];
  if constexpr (VEC) {
    const float4 v = *reinterpret_cast<const float4*>(x + e);
    *reinterpret_cast<float4*>(y + e) =
        make_float4((v.x - st.x) * st.y, (v.y - st.x) * st.y, (v.z - st.x) * st.y, (v.w - st.x) * st.y);
  } else {
    y[e] = (x[e] - st.x) * st.y;
  }
}

// ---------------------------------------------- stride-4 conv weight repacks
// down: Wd[o][t*C + i] = w[o][i][t]; up: Wu[t*C + o][i] = w[i][o][t] (bf16 bits)
__global__ void __launch_bounds__(256) repack_down_kernel(const uint16_t* __restrict__ w, uint16_t* __restrict__ out,
                                                          int C) {
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= 4LL * C * C) return;
  const long long o = idx / (4LL * C);
  const long long rem = idx - o * 4LL * C;
  const int t = static_cast<int>(rem / C);
  const long long i = rem - static_cast<long long>(t) * C;
  out[idx] = w[(o * C + i) * 4 + t];
}

__global__ void __launch_bounds__(256) repack_up_kernel(const uint16_t* __restrict__ w, uint16_t* __restrict__ out,
                                                        const uint16_t* __restrict__ b, uint16_t* __restrict__ b4,
                                                        int C) {
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx < 4LL * C && b != nullptr) b4[idx] = b[idx % C];
  if (idx >= 4LL * C * C) return;
  const long long r = idx / C;  // t*C + o
  const long long i = idx - r * C;
  const int t = static_cast<int>(r / C);
  const long long o = r - static_cast<long long>(t) * C;
  out[idx] = w[(i * C + o) * 4 + t];
}

// --------------------------------------------------------------- EMA stats
// Counting sort of rows by code: histogram, exclusive scan (one block), then a
// stable scatter (each code's rows in increasing row index), then one warp
// per code sums its rows in that order.
__global__ void __launch_bounds__(256) code_histogram_kernel(const int32_t* __restrict__ codes, long long N, int K,
                                                             int* __restrict__ hist, int* __restrict__ err) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= N) return;
  const int c = codes[i];
  if (c < 0 || c >= K) {
    atomicOr(err, kErrBadIndex);
    return;
  }
  atomicAdd(hist + c, 1);
}

__global__ void __launch_bounds__(1024) exclusive_scan_kernel(const int* __restrict__ hist, int* __restrict__ start,
                                                              int K) {
  // one block: each thread scans a contiguous slice, then the slice totals
  __shared__ int part[1024];
  const int per = (K + blockDim.x - 1) / blockDim.x;
  const int lo = threadIdx.x * per, hi = min(lo + per, K);
  int sum = 0;
  for (int k = lo; k < hi; ++k) sum += hist[k];
  part[threadIdx.x] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int t = 0; t < static_cast<int>(blockDim.x); ++t) {
      const int v = part[t];
      part[t] = run;
      run += v;
    }
  }
  __syncthreads();
  int run = part[threadIdx.x];
  for (int k = lo; k < hi; ++k) {
    start[k] = run;
    run += hist[k];
  }
  if (threadIdx.x == blockDim.x - 1) start[K] = run;
}

// Stable scatter in three steps: rows are cut into chunks, each chunk's code
// histogram gives every (chunk, code) its first slot after the code's start
// and the earlier chunks' rows, and one warp per chunk then walks its rows in
// order placing each at its slot (lanes with the same code ranked by lane).
__global__ void __launch_bounds__(256) chunk_histogram_kernel(const int32_t* __restrict__ codes, long long N,
                                                              int K, int chunk, int* __restrict__ chunk_hist) {
  // block c counts the codes of rows [c*chunk, (c+1)*chunk) into chunk_hist[c*K + k]
  const long long r0 = static_cast<long long>(blockIdx.x) * chunk;
  for (long long i = r0 + threadIdx.x; i < min(r0 + chunk, N); i += blockDim.x) {
    const int c = codes[i];
    if (c >= 0 && c < K) atomicAdd(chunk_hist + static_cast<size_t>(blockIdx.x) * K + c, 1);
  }
}

// offsets[c*K + k] = start[k] + sum over earlier chunks of their count of k
__global__ void __launch_bounds__(256) chunk_offsets_kernel(const int* __restrict__ chunk_hist,
                                                            const int* __restrict__ start, int nchunks, int K,
                                                            int* __restrict__ offsets) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= K) return;
  int run = start[k];
  for (int c = 0; c < nchunks; ++c) {
    offsets[static_cast<size_t>(c) * K + k] = run;
    run += chunk_hist[static_cast<size_t>(c) * K + k];
  }
}

// one warp per chunk walks its rows in order; lane-parallel ballots give each
// row its rank among the chunk's earlier rows with the same code
__global__ void __launch_bounds__(32) chunk_scatter_kernel(const int32_t* __restrict__ codes, long long N, int K,
                                                           int chunk, int* __restrict__ offsets,
                                                           int* __restrict__ order) {
  const int lane = threadIdx.x;
  const long long r0 = static_cast<long long>(blockIdx.x) * chunk;
  int* off = offsets + static_cast<size_t>(blockIdx.x) * K;
  for (long long base = r0; base < min(r0 + chunk, N); base += 32) {
    const long long i = base + lane;
    const bool valid = i < min(r0 + chunk, N);
    const int c = valid ? codes[i] : -1;
    const bool ok = valid && c >= 0 && c < K;
    // rank among lanes < lane with the same code, then the first such lane bumps the offset
    const unsigned same = __match_any_sync(0xffffffffu, ok ? c : -1);
    const int rank = __popc(same & ((1u << lane) - 1u));
    const int cnt = __popc(same);
    int pos = 0;
    if (ok && rank == 0) pos = off[c];
    pos = __shfl_sync(0xffffffffu, pos, __ffs(same) - 1);
    if (ok) order[pos + rank] = static_cast<int>(i);
    __syncwarp();
    if (ok && rank == 0) off[c] = pos + cnt;
    __syncwarp();
  }
}

// counts[k] = rows of code k; sums[k, :] = their rows of u summed in row order (f32)
__global__ void __launch_bounds__(256) code_sums_kernel(const float* __restrict__ u, const int* __restrict__ order,
                                                        const int* __restrict__ start, int K, int D,
                                                        float* __restrict__ counts, float* __restrict__ sums) {
  const int k = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (k >= K) return;
  const int a = start[k], b = start[k + 1];
  if (lane == 0) counts[k] = static_cast<float>(b - a);
  for (int d = lane * 4; d < D; d += 128) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = a; j < b; ++j) {
      const float4 v = *reinterpret_cast<const float4*>(u + static_cast<size_t>(order[j]) * D + d);
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    *reinterpret_cast<float4*>(sums + static_cast<size_t>(k) * D + d) = acc;
  }
}

// N <- g N + (1-g) n; n_tot = sum N (f64, one block); N_hat = (N + eps) / (n_tot + K eps) * n_tot;
// m <- g m + (1-g) s; e = m / N_hat (f32, and bf16 bits)
__global__ void __launch_bounds__(1024) ema_counts_kernel(float* __restrict__ Nk, const float* __restrict__ n, int K,
                                                          float gamma, float eps, float* __restrict__ nhat) {
  __shared__ double red[32];
  double s = 0.0;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const float v = gamma * Nk[k] + (1.f - gamma) * n[k];
    Nk[k] = v;
    s += v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  __shared__ float tot;
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += red[w];
    tot = static_cast<float>(t);
  }
  __syncthreads();
  const float nt = tot;
  for (int k = threadIdx.x; k < K; k += blockDim.x) nhat[k] = (Nk[k] + eps) / (nt + K * eps) * nt;
}

__global__ void __launch_bounds__(256) ema_embed_kernel(float* __restrict__ m, const float* __restrict__ s,
                                                        const float* __restrict__ nhat, long long KD, int D,
                                                        float gamma, float* __restrict__ e_f32,
                                                        uint16_t* __restrict__ e_bf16) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= KD) return;
  const float v = gamma * m[i] + (1.f - gamma) * s[i];
  m[i] = v;
  const float e = v / nhat[i / D];
  if (e_f32 != nullptr) e_f32[i] = e;
  if (e_bf16 != nullptr) e_bf16[i] = f32_to_bf16(e);
}

int check_ctx_aux(ncm_ctx* ctx) {
  if (ctx == nullptr) return ncm_fail(NCM_EINVAL, "null context");
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev != ctx->device) {
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e != cudaSuccess) return ncm_set_cuda_error(e);
  }
  return NCM_OK;
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace ncm

using namespace ncm;

extern "C" {

int ncm_group_norm(ncm_ctx_t* ctx, const float* x, float* y, int64_t batch, int64_t T, int64_t C, int32_t groups,
                   float eps, ncm_stream_t stream) {
  int rc = check_ctx_aux(ctx);
  if (rc) return rc;
  if (batch <= 0 || T <= 0 || C <= 0 || groups <= 0 || C % groups != 0 || batch * groups > INT32_MAX ||
      T > INT32_MAX || C > INT32_MAX)
    return ncm_fail(NCM_EINVAL, "group_norm: bad shape (B=%lld T=%lld C=%lld groups=%d)", (long long)batch,
                    (long long)T, (long long)C, groups);
  if (!x || !y) return ncm_fail(NCM_EINVAL, "group_norm: null buffer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int n_sg = static_cast<int>(batch * groups);
  WsCarver cv;
  const size_t o_part = cv.take(sizeof(double2) * n_sg * kGnChunks), o_stat = cv.take(sizeof(float2) * n_sg);
  uint8_t* ws = static_cast<uint8_t*>(ctx_workspace(ctx, cv.offset));
  if (ws == nullptr) return ncm_fail(NCM_ENOMEM, "group_norm: workspace allocation failed");
  double2* part = reinterpret_cast<double2*>(ws + o_part);
  float2* stat = reinterpret_cast<float2*>(ws + o_stat);
  Launch _launch(ctx, KID_DECODER_ELEMENTWISE, st);
  const bool vec = (C / groups) % 4 == 0 && al16(x) && al16(y);
  if (vec)
    group_norm_partial_kernel<true><<<dim3(n_sg, kGnChunks), 256, 0, st>>>(x, static_cast<int>(T),
                                                                           static_cast<int>(C), groups, part);
  else
    group_norm_partial_kernel<false><<<dim3(n_sg, kGnChunks), 256, 0, st>>>(x, static_cast<int>(T),
                                                                            static_cast<int>(C), groups, part);
  group_norm_stats_kernel<<<blocks_of(n_sg, 256), 256, 0, st>>>(part, n_sg, T * (C / groups), eps, stat);
  const long long n = batch * T * C;
  if (vec)
    group_norm_apply_kernel<true><<<blocks_of(n / 4, 256), 256, 0, st>>>(x, y, n, static_cast<int>(T),
                                                                         static_cast<int>(C), groups, stat);
  else
    group_norm_apply_kernel<false><<<blocks_of(n, 256), 256, 0, st>>>(x, y, n, static_cast<int>(T),
                                                                      static_cast<int>(C), groups, stat);
  NCM_CUDA_TRY(cudaGetLastError());
  return NCM_OK;
}

int ncm_conv_down4(ncm_ctx_t* ctx, const uint16_t* x, const uint16_t* weight, const uint16_t* bias, uint16_t* y,
                   int64_t batch, int64_t L, int64_t C, ncm_stream_t stream) {
  int rc = check_ctx_aux(ctx);
  if (rc) return rc;
  if (batch <= 0 || L <= 0 || L % 4 != 0 || C <= 0 || C % 8 != 0 || batch * L > INT32_MAX)
    return ncm_fail(NCM_EINVAL, "conv_down4: bad shape (B=%lld L=%lld C=%lld; L %% 4 == 0, C %% 8 == 0)",
                    (long long)batch, (long long)L, (long long)C);
  if (!x || !weight || !y) return ncm_fail(NCM_EINVAL, "conv_down4: null buffer");
  if (!al16(x) || !al16(weight) || !al16(y) || (bias && !al16(bias)))
    return ncm_fail(NCM_EINVAL, "conv_down4: buffers must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint16_t* wd = static_cast<uint16_t*>(ctx_workspace(ctx, 2 * 4 * C * C));
  if (wd == nullptr) return ncm_fail(NCM_ENOMEM, "conv_down4: workspace allocation failed");
  {
    Launch _launch(ctx, KID_CAST, st);
    repack_down_kernel<<<blocks_of(4 * C * C, 256), 256, 0, st>>>(weight, wd, static_cast<int>(C));
    NCM_CUDA_TRY(cudaGetLastError());
  }
  // four consecutive rows form one row of 4C values
  return linear_bf16(ctx, x, wd, bias, y, nullptr, batch * L / 4, 4 * C, C, st);
}

int ncm_conv_up4(ncm_ctx_t* ctx, const uint16_t* x, const uint16_t* weight, const uint16_t* bias, uint16_t* y,
                 int64_t batch, int64_t L, int64_t C, ncm_stream_t stream) {
  int rc = check_ctx_aux(ctx);
  if (rc) return rc;
  if (batch <= 0 || L <= 0 || C <= 0 || C % 8 != 0 || batch * L * 4 > INT32_MAX)
    return ncm_fail(NCM_EINVAL, "conv_up4: bad shape (B=%lld L=%lld C=%lld; C %% 8 == 0)", (long long)batch,
                    (long long)L, (long long)C);
  if (!x || !weight || !y) return ncm_fail(NCM_EINVAL, "conv_up4: null buffer");
  if (!al16(x) || !al16(weight) || !al16(y) || (bias && !al16(bias)))
    return ncm_fail(NCM_EINVAL, "conv_up4: buffers must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  WsCarver cv;
  const size_t o_w = cv.take(2 * 4 * C * C), o_b = cv.take(2 * 4 * C);
  uint8_t* ws = static_cast<uint8_t*>(ctx_workspace(ctx, cv.offset));
  if (ws == nullptr) return ncm_fail(NCM_ENOMEM, "conv_up4: workspace allocation failed");
  uint16_t* wu = reinterpret_cast<uint16_t*>(ws + o_w);
  uint16_t* b4 = bias ? reinterpret_cast<uint16_t*>(ws + o_b) : nullptr;
  {
    Launch _launch(ctx, KID_CAST, st);
    repack_up_kernel<<<blocks_of(4 * C * C, 256), 256, 0, st>>>(weight, wu, bias, b4, static_cast<int>(C));
    NCM_CUDA_TRY(cudaGetLastError());
  }
  // output row j of 4C values is output positions 4j .. 4j+3
  return linear_bf16(ctx, x, wu, b4, y, nullptr, batch * L, C, 4 * C, st);
}

int ncm_ema_code_stats(ncm_ctx_t* ctx, const float* u, const int32_t* codes, float* counts, float* sums, int64_t N,
                       int64_t D, int64_t K, ncm_stream_t stream) {
  int rc = check_ctx_aux(ctx);
  if (rc) return rc;
  if (N <= 0 || D <= 0 || D % 4 != 0 || K <= 0 || N > INT32_MAX || K > INT32_MAX / 2)
    return ncm_fail(NCM_EINVAL, "ema_code_stats: bad shape (N=%lld D=%lld K=%lld; D %% 4 == 0)", (long long)N,
                    (long long)D, (long long)K);
  if (!u || !codes || !counts || !sums) return ncm_fail(NCM_EINVAL, "ema_code_stats: null buffer");
  if (!al16(u) || !al16(sums)) return ncm_fail(NCM_EINVAL, "ema_code_stats: u and sums must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // about 256 chunks (one scatter warp each), at least 256 rows per chunk
  const int chunk = static_cast<int>(std::max<int64_t>(256, ((N + 255) / 256 + 31) / 32 * 32));
  const int nchunks = static_cast<int>((N + chunk - 1) / chunk);
  WsCarver cv;
  const size_t o_hist = cv.take(sizeof(int) * K), o_start = cv.take(sizeof(int) * (K + 1));
  const size_t o_ch = cv.take(sizeof(int) * static_cast<size_t>(nchunks) * K);
  const size_t o_off = cv.take(sizeof(int) * static_cast<size_t>(nchunks) * K);
  const size_t o_order = cv.take(sizeof(int) * N);
  uint8_t* ws = static_cast<uint8_t*>(ctx_workspace(ctx, cv.offset));
  if (ws == nullptr) return ncm_fail(NCM_ENOMEM, "ema_code_stats: workspace allocation failed");
  int* hist = reinterpret_cast<int*>(ws + o_hist);
  int* start = reinterpret_cast<int*>(ws + o_start);
  int* chist = reinterpret_cast<int*>(ws + o_ch);
  int* offs = reinterpret_cast<int*>(ws + o_off);
  int* order = reinterpret_cast<int*>(ws + o_order);
  NCM_CUDA_TRY(cudaMemsetAsync(hist, 0, sizeof(int) * K, st));
  NCM_CUDA_TRY(cudaMemsetAsync(chist, 0, sizeof(int) * static_cast<size_t>(nchunks) * K, st));
  Launch _launch(ctx, KID_SCALE_UPDATE, st);
  code_histogram_kernel<<<blocks_of(N, 256), 256, 0, st>>>(codes, N, static_cast<int>(K), hist, ctx->d_err);
  exclusive_scan_kernel<<<1, 1024, 0, st>>>(hist, start, static_cast<int>(K));
  chunk_histogram_kernel<<<nchunks, 256, 0, st>>>(codes, N, static_cast<int>(K), chunk, chist);
  chunk_offsets_kernel<<<blocks_of(K, 256), 256, 0, st>>>(chist, start, nchunks, static_cast<int>(K), offs);
  chunk_scatter_kernel<<<nchunks, 32, 0, st>>>(codes, N, static_cast<int>(K), chunk, offs, order);
  code_sums_kernel<<<blocks_of(K, 8), 256, 0, st>>>(u, order, start, static_cast<int>(K), static_cast<int>(D), counts,
                                                     sums);
  NCM_CUDA_TRY(cudaGetLastError());
  return NCM_OK;
}

int ncm_ema_update(ncm_ctx_t* ctx, const float* counts, const float* sums, float* ema_count, float* ema_sum,
                   float* codebook_f32, uint16_t* codebook_bf16, int64_t K, int64_t D, float decay, float eps,
                   ncm_stream_t stream) {
  int rc = check_ctx_aux(ctx);
  if (rc) return rc;
  if (K <= 0 || D <= 0 || K * D > (1LL << 40) || !(decay >= 0.f && decay <= 1.f) || !(eps >= 0.f))
    return ncm_fail(NCM_EINVAL, "ema_update: bad arguments");
  if (!counts || !sums || !ema_count || !ema_sum) return ncm_fail(NCM_EINVAL, "ema_update: null buffer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float* nhat = static_cast<float*>(ctx_workspace(ctx, sizeof(float) * K));
  if (nhat == nullptr) return ncm_fail(NCM_ENOMEM, "ema_update: workspace allocation failed");
  Launch _launch(ctx, KID_SCALE_UPDATE, st);
  ema_counts_kernel<<<1, 1024, 0, st>>>(ema_count, counts, static_cast<int>(K), decay, eps, nhat);
  ema_embed_kernel<<<blocks_of(K * D, 256), 256, 0, st>>>(ema_sum, sums, nhat, K * D, static_cast<int>(D), decay,
                                                           codebook_f32, codebook_bf16);
  NCM_CUDA_TRY(cudaGetLastError());
  return NCM_OK;
}

}  // extern "C"
