// Kernel-3 convolution along time and time upsampling (R5 modes, and the
// quantiser's residual convolutions):
//
//  * upsampling q [B, Tq, D] -> [B, T, D] as F.interpolate(size=T) does it,
//    nearest or linear (align_corners=False) — the U_i of
//    research/reference/vq_forward_semantics.md:82 and :108 (`_up_to_full`);
//  * the Conv1d(D, D, kernel 3, padding 1) of `apply_post_upsample_conv`
//    (src/ncm_model.zig:296-326: out = x + bias + conv(x)) and of the
//    quantiser's Phi (vq_forward_semantics.md:93-100: out = (1-r) h + r Conv(h)),
//    both as val = alpha * x + beta * (bias + conv(x)) per row segment.
//
// The convolution is an implicit GEMM on the tcgen05 linear kernel: the input
// is copied once to bf16 in "padded" row order (a zero row around every
// segment, zero columns up to a multiple of 64), the [D, D, 3] kernel is
// repacked tap-major to [D, 3 * dp], and K-chunk k of the GEMM reads the A
// rows shifted by its tap. The epilogue applies the blend and scatters rows
// back to the unpadded order (gemm.cu, mode 3).
#include <algorithm>
#include <vector>

#include "internal.h"

namespace ncm {
namespace {

// [o][i][tap] -> [o][tap][i] (i padded to dp with zeros), rounded to bf16.
__global__ void __launch_bounds__(256) conv_repack_kernel(const uint16_t* __restrict__ w_bf16,
                                                          const float* __restrict__ w_f32, uint16_t* __restrict__ out,
                                                          long long width, long long dp) {
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total = width * 3 * dp;
  if (idx >= total) return;
  const long long o = idx / (3 * dp);
  const long long rem = idx - o * 3 * dp;
  const int tap = static_cast<int>(rem / dp);
  const long long i = rem - tap * dp;
  uint16_t v = 0;
  if (i < width) {
    const long long src = (o * width + i) * 3 + tap;
    v = w_bf16 != nullptr ? w_bf16[src] : f32_to_bf16(w_f32[src]);
  }
  out[idx] = v;
}

// padded row p, 4 columns per thread: bf16(x[real row]) or zeros.
__global__ void __launch_bounds__(256) conv_pad_kernel(const float* __restrict__ x_f32,
                                                       const uint16_t* __restrict__ x_bf16, uint16_t* __restrict__ out,
                                                       const SegMap map, long long width, long long dp) {
  const long long g4 = dp / 4;
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long Mp = map.padded_rows();
  if (idx >= Mp * g4) return;
  const long long p = idx / g4;
  const long long c = (idx - p * g4) * 4;
  const long long r = map.real_row(p);
  float v[4] = {0.f, 0.f, 0.f, 0.f};
  if (r >= 0) {
    const size_t base = static_cast<size_t>(r) * width;
    for (int j = 0; j < 4; ++j) {
      if (c + j >= width) break;
      v[j] = x_f32 != nullptr ? x_f32[base + c + j] : bf16_to_f32(x_bf16[base + c + j]);
    }
  }
  *reinterpret_cast<uint2*>(out + p * dp + c) = make_uint2(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]));
}

// One thread per (output row, 4 channels). Nearest: src = min(floor(t * s), Tq - 1).
// Linear (align_corners=False): src = max(fma(s, t + 0.5, -0.5), 0),
// i0 = trunc(src), l1 = src - i0, l0 = 1 - l1, i1 = min(i0 + 1, Tq - 1),
// Q = fma(q[i0], l0, q[i1] * l1) — the operation order of PyTorch's CPU
// kernel, so the values match it bit for bit. s = float(Tq) / float(T).
__global__ void __launch_bounds__(256) upsample_kernel(const float* __restrict__ q, long long B, long long Tq,
                                                       long long T, int D, int mode, float s,
                                                       float* __restrict__ out_f32, uint16_t* __restrict__ out_pad,
                                                       long long dp, float* __restrict__ resid,
                                                       float* __restrict__ acc) {
  const int d4 = D / 4;
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= B * T * d4) return;
  const long long row = idx / d4;
  const int d = static_cast<int>(idx - row * d4) * 4;
  const long long b = row / T;
  const long long t = row - b * T;
  const float* qb = q + static_cast<size_t>(b) * Tq * D;
  float4 Q;
  if (mode == 0) {
    long long i0 = static_cast<long long>(floorf(__fmul_rn(static_cast<float>(t), s)));
    if (i0 > Tq - 1) i0 = Tq - 1;
    Q = *reinterpret_cast<const float4*>(qb + i0 * D + d);
  } else {
    float src = __fmaf_rn(s, static_cast<float>(t) + 0.5f, -0.5f);
    src = fmaxf(src, 0.f);
    const long long i0 = static_cast<long long>(src);
    const float l1 = fminf(fmaxf(src - static_cast<float>(i0), 0.f), 1.f);
    const float l0 = 1.f - l1;
    const long long i1 = i0 < Tq - 1 ? i0 + 1 : i0;
    const float4 a = *reinterpret_cast<const float4*>(qb + i0 * D + d);
    const float4 c = *reinterpret_cast<const float4*>(qb + i1 * D + d);
    Q.x = __fmaf_rn(a.x, l0, __fmul_rn(c.x, l1));
    Q.y = __fmaf_rn(a.y, l0, __fmul_rn(c.y, l1));
    Q.z = __fmaf_rn(a.z, l0, __fmul_rn(c.z, l1));
    Q.w = __fmaf_rn(a.w, l0, __fmul_rn(c.w, l1));
  }
  const size_t o = static_cast<size_t>(row) * D + d;
  if (out_f32 != nullptr) *reinterpret_cast<float4*>(out_f32 + o) = Q;
  if (resid != nullptr) {
    float4 r = *reinterpret_cast<const float4*>(resid + o);
    r.x -= Q.x;
    r.y -= Q.y;
    r.z -= Q.z;
    r.w -= Q.w;
    *reinterpret_cast<float4*>(resid + o) = r;
  }
  if (acc != nullptr) {
    float4 a = *reinterpret_cast<const float4*>(acc + o);
    a.x += Q.x;
    a.y += Q.y;
    a.z += Q.z;
    a.w += Q.w;
    *reinterpret_cast<float4*>(acc + o) = a;
  }
  if (out_pad != nullptr) {
    // segments of T rows: padded row of (b, t) is b * (T + 1) + 1 + t
    const bool last = d + 4 == D;
    const long long p = b * (T + 1) + 1 + t;
    *reinterpret_cast<uint2*>(out_pad + p * dp + d) = make_uint2(pack_bf16x2(Q.x, Q.y), pack_bf16x2(Q.z, Q.w));
    if (last)
      for (long long c = D; c < dp; ++c) out_pad[p * dp + c] = 0;
    // the zero row before this item, and after the last one
    long long zrows[2] = {-1, -1};
    if (t == 0) zrows[0] = b * (T + 1);
    if (b == B - 1 && t == T - 1) zrows[1] = B * (T + 1);
    for (int z = 0; z < 2; ++z) {
      if (zrows[z] < 0) continue;
      *reinterpret_cast<uint2*>(out_pad + zrows[z] * dp + d) = make_uint2(0u, 0u);
      if (last)
        for (long long c = D; c < dp; ++c) out_pad[zrows[z] * dp + c] = 0;
    }
  }
}

int blocks_for(long long n) { return static_cast<int>((n + 255) / 256); }

}  // namespace

bool make_segmap(SegMap* m, int64_t rows, int nseg, const int64_t* lengths) {
  *m = SegMap{};
  if (lengths != nullptr && (nseg <= 0 || (nseg == 1 && lengths[0] != rows))) return false;
  if (lengths == nullptr || nseg == 1) {
    m->seg_len = static_cast<int>(rows);
    m->nseg = 1;
    return rows > 0 && rows <= INT32_MAX / 2;
  }
  bool uniform = true;
  int64_t sum = 0;
  for (int s = 0; s < nseg; ++s) {
    if (lengths[s] <= 0) return false;
    uniform = uniform && lengths[s] == lengths[0];
    sum += lengths[s];
  }
  if (sum != rows || rows + nseg + 1 > INT32_MAX / 2) return false;
  m->nseg = nseg;
  if (uniform) {
    m->seg_len = static_cast<int>(lengths[0]);
    return true;
  }
  if (nseg > kMaxConvSegments) return false;
  m->seg_len = 0;
  int64_t at = 0;
  for (int s = 0; s < nseg; ++s) {
    m->rstart[s] = static_cast<int>(at);
    at += lengths[s];
  }
  m->rstart[nseg] = static_cast<int>(at);
  return true;
}

cudaError_t launch_conv_repack(const uint16_t* w_bf16, const float* w_f32, uint16_t* out, int64_t width, int64_t dp,
                               cudaStream_t stream) {
  const long long total = width * 3 * dp;
  conv_repack_kernel<<<blocks_for(total), 256, 0, stream>>>(w_bf16, w_f32, out, width, dp);
  return cudaGetLastError();
}

cudaError_t launch_conv_pad(const float* x_f32, const uint16_t* x_bf16, uint16_t* out, const SegMap& map,
                            int64_t width, int64_t dp, cudaStream_t stream) {
  const long long n = map.padded_rows() * (dp / 4);
  conv_pad_kernel<<<blocks_for(n), 256, 0, stream>>>(x_f32, x_bf16, out, map, width, dp);
  return cudaGetLastError();
}

cudaError_t launch_upsample(const float* q, int64_t B, int64_t Tq, int64_t T, int64_t D, int mode, float* out_f32,
                            uint16_t* out_pad, int64_t dp, float* resid, float* acc, cudaStream_t stream) {
  const float s = static_cast<float>(Tq) / static_cast<float>(T);
  const long long n = B * T * (D / 4);
  upsample_kernel<<<blocks_for(n), 256, 0, stream>>>(q, B, Tq, T, static_cast<int>(D), mode, s, out_f32, out_pad,
                                                     dp, resid, acc);
  return cudaGetLastError();
}

}  // namespace ncm

using namespace ncm;

namespace {

bool a4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }
bool a16c(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int conv_ctx_ok(ncm_ctx* ctx) {
  if (ctx == nullptr) return ncm_fail(NCM_EINVAL, "null context");
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev != ctx->device) {
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e != cudaSuccess) return ncm_set_cuda_error(e);
  }
  return NCM_OK;
}

int64_t pad64(int64_t w) { return (w + 63) / 64 * 64; }

// Workspace regions of one convolution: the padded bf16 input and the packed kernel.
struct ConvWs {
  size_t o_pad, o_w;
};
ConvWs carve_conv(WsCarver& cv, const SegMap& map, int64_t width) {
  const int64_t dp = pad64(width);
  ConvWs c;
  c.o_pad = cv.take(2 * map.padded_rows() * dp);
  c.o_w = cv.take(2 * width * 3 * dp);
  return c;
}

// Shared body: conv over device buffers; `w_bf16` or `w_f32` holds the [width, width, 3] kernel.
int conv_device(ncm_ctx* ctx, uint8_t* ws, const ConvWs& cw, const float* x, const uint16_t* w_bf16,
                const float* w_f32, const float* bias, float* out, int64_t width, const SegMap& map, float alpha,
                float beta, cudaStream_t st) {
  const int64_t dp = pad64(width);
  uint16_t* a_pad = reinterpret_cast<uint16_t*>(ws + cw.o_pad);
  uint16_t* w_pack = reinterpret_cast<uint16_t*>(ws + cw.o_w);
  {
    Launch _launch(ctx, KID_CAST, st);
    NCM_CUDA_TRY(launch_conv_repack(w_bf16, w_f32, w_pack, width, dp, st));
  }
  {
    Launch _launch(ctx, KID_CAST, st);
    NCM_CUDA_TRY(launch_conv_pad(x, nullptr, a_pad, map, width, dp, st));
  }
  ConvEpilogue ep{};
  ep.x_f32 = x;
  ep.out_f32 = out;
  ep.bias = bias;
  ep.alpha = alpha;
  ep.beta = beta;
  return conv3_gemm(ctx, a_pad, w_pack, map, dp, width, ep, st);
}

}  // namespace

extern "C" {

int ncm_upsample(ncm_ctx_t* ctx, const float* q, float* out, int64_t batch, int64_t in_len, int64_t out_len,
                 int64_t width, int32_t mode, ncm_stream_t stream) {
  int rc = conv_ctx_ok(ctx);
  if (rc) return rc;
  if (batch <= 0 || in_len <= 0 || out_len <= 0 || width <= 0 || width % 4 != 0 || (mode != 0 && mode != 1))
    return ncm_fail(NCM_EINVAL, "upsample: bad arguments (B=%lld in=%lld out=%lld width=%lld mode=%d)",
                    (long long)batch, (long long)in_len, (long long)out_len, (long long)width, mode);
  if (!q || !out || !a16c(q) || !a16c(out)) return ncm_fail(NCM_EINVAL, "upsample: buffers must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Launch _launch(ctx, KID_UPSAMPLE, st);
  NCM_CUDA_TRY(launch_upsample(q, batch, in_len, out_len, width, mode, out, nullptr, 0, nullptr, nullptr, st));
  return NCM_OK;
}

int ncm_conv1d_k3(ncm_ctx_t* ctx, const float* x, const uint16_t* weight, const float* bias, float* out,
                  int64_t rows, int64_t width, int32_t num_segments, const int64_t* segment_lengths, float alpha,
                  float beta, ncm_stream_t stream) {
  int rc = conv_ctx_ok(ctx);
  if (rc) return rc;
  if (rows <= 0 || width <= 0 || width > INT32_MAX / 4)
    return ncm_fail(NCM_EINVAL, "conv: bad shape rows=%lld width=%lld", (long long)rows, (long long)width);
  if (!x || !weight || !out) return ncm_fail(NCM_EINVAL, "conv: null buffer");
  if (!a4(x) || !a4(out) || (bias && !a4(bias)) || (reinterpret_cast<uintptr_t>(weight) & 1u))
    return ncm_fail(NCM_EINVAL, "conv: misaligned buffer");
  SegMap map;
  if (!make_segmap(&map, rows, segment_lengths ? num_segments : 1, segment_lengths))
    return ncm_fail(NCM_EINVAL,
                    "conv: segment lengths must be positive and sum to rows (at most %d segments of unequal length)",
                    kMaxConvSegments);
  WsCarver cv;
  const ConvWs cw = carve_conv(cv, map, width);
  uint8_t* ws = static_cast<uint8_t*>(ctx_workspace(ctx, cv.offset));
  if (ws == nullptr) return ncm_fail(NCM_ENOMEM, "conv: workspace allocation failed");
  return conv_device(ctx, ws, cw, x, weight, nullptr, bias, out, width, map, alpha, beta,
                     static_cast<cudaStream_t>(stream));
}

int ncm_post_upsample_conv_host_f32(ncm_ctx_t* ctx, float* input, const float* weight, const float* bias,
                                    int64_t row_count, int64_t width) {
  int rc = conv_ctx_ok(ctx);
  if (rc) return rc;
  if (row_count <= 0 || width <= 0 || width > INT32_MAX / 4)
    return ncm_fail(NCM_EINVAL, "post_upsample_conv: bad shape rows=%lld width=%lld", (long long)row_count,
                    (long long)width);
  if (!input || !weight || !bias) return ncm_fail(NCM_EINVAL, "post_upsample_conv: null buffer");
  SegMap map;
  if (!make_segmap(&map, row_count, 1, nullptr)) return ncm_fail(NCM_EINVAL, "post_upsample_conv: too many rows");
  WsCarver cv;
  const size_t o_x = cv.take(sizeof(float) * row_count * width);
  const size_t o_w = cv.take(sizeof(float) * width * width * 3);
  const size_t o_b = cv.take(sizeof(float) * width);
  const ConvWs cw = carve_conv(cv, map, width);
  uint8_t* ws = static_cast<uint8_t*>(ctx_workspace(ctx, cv.offset));
  if (ws == nullptr) return ncm_fail(NCM_ENOMEM, "post_upsample_conv: workspace allocation failed");
  float* xd = reinterpret_cast<float*>(ws + o_x);
  float* wd = reinterpret_cast<float*>(ws + o_w);
  float* bd = reinterpret_cast<float*>(ws + o_b);
  cudaStream_t st = 0;
  NCM_CUDA_TRY(cudaMemcpyAsync(xd, input, sizeof(float) * row_count * width, cudaMemcpyHostToDevice, st));
  NCM_CUDA_TRY(cudaMemcpyAsync(wd, weight, sizeof(float) * width * width * 3, cudaMemcpyHostToDevice, st));
  NCM_CUDA_TRY(cudaMemcpyAsync(bd, bias, sizeof(float) * width, cudaMemcpyHostToDevice, st));
  // in place: the epilogue reads x[row] before writing out[row], and the GEMM reads the padded copy
  rc = conv_device(ctx, ws, cw, xd, nullptr, wd, bd, xd, width, map, 1.f, 1.f, st);
  if (rc) return rc;
  NCM_CUDA_TRY(cudaMemcpyAsync(input, xd, sizeof(float) * row_count * width, cudaMemcpyDeviceToHost, st));
  NCM_CUDA_TRY(cudaStreamSynchronize(st));
  return NCM_OK;
}

}  // extern "C"
