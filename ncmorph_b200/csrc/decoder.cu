// NCM decoder forward on the GPU (config 4): the bf16 layer of ncmorph's
// decoder (src/decoder.zig:168-216, bf16 mode) driven by the NCM input
// assembly of src/ncm_model.zig:89-250 — input projection, level embedding,
// per-level restarting RoPE positions, block-diagonal or block-causal mask.
//
// Elementwise kernels here restate the reference's bf16-mode rounding points
// exactly (RMSNorm root.zig:243-252, rotate_head :615-633, SiLU :264-269,
// residual adds decoder.zig:310-313); the projections run on the tcgen05
// linear and attention on the fused tcgen05 attention kernel.
#include <cmath>
#include <cstring>
#include <vector>

#include "internal.h"
#include "ptx.cuh"

namespace ncm {
namespace {

// ---------------------------------------------------------------- RMSNorm
// One warp per row. y = bf16(bf16(x * inv) * bf16(w)) (+ bias, rounded),
// inv = 1 / sqrt(mean(x^2) + eps) in f32. NCH > 0: the row (at most NCH * 256
// columns) is read once into registers; NCH = 0: any width, read twice.
// Rounding is the hardware round-to-nearest-even (the reference rule for
// every non-NaN value).
template <int NCH>
__global__ void __launch_bounds__(256) rms_norm_bf16_kernel(const uint16_t* __restrict__ x,
                                                            const uint16_t* __restrict__ w,
                                                            const uint16_t* __restrict__ bias,
                                                            uint16_t* __restrict__ y, int rows, int width,
                                                            float eps) {
  pdl_wait();
  pdl_launch_dependents();
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const uint16_t* xr = x + static_cast<size_t>(row) * width;
  constexpr int REG = NCH > 0 ? NCH : 1;
  uint4 keep[REG];
  float ss = 0.f;
  auto add_sq = [&ss](const uint4& v) {
    const uint32_t p[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float a = bf16lo(p[e]), b = bf16hi(p[e]);
      ss = fmaf(a, a, ss);
      ss = fmaf(b, b, ss);
    }
  };
  if constexpr (NCH > 0) {
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int i = c * 256 + lane * 8;
      keep[c] = i < width ? *reinterpret_cast<const uint4*>(xr + i) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int c = 0; c < NCH; ++c) add_sq(keep[c]);
  } else {
    for (int i = lane * 8; i < width; i += 256) add_sq(*reinterpret_cast<const uint4*>(xr + i));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float ms = ss / static_cast<float>(width);
  const float inv = 1.0f / sqrtf(ms + eps);
  uint16_t* yr = y + static_cast<size_t>(row) * width;
  auto emit = [&](int i, const uint4& v) {
    const uint4 wv = __ldg(reinterpret_cast<const uint4*>(w + i));
    uint4 bv = make_uint4(0, 0, 0, 0);
    if (bias != nullptr) bv = __ldg(reinterpret_cast<const uint4*>(bias + i));
    const uint32_t p[4] = {v.x, v.y, v.z, v.w};
    const uint32_t q[4] = {wv.x, wv.y, wv.z, wv.w};
    const uint32_t r[4] = {bv.x, bv.y, bv.z, bv.w};
    uint32_t o4[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint32_t n = cvt_bf16x2(bf16lo(p[e]) * inv, bf16hi(p[e]) * inv);
      const uint32_t m = cvt_bf16x2(bf16lo(n) * bf16lo(q[e]), bf16hi(n) * bf16hi(q[e]));
      if (bias != nullptr)
        o4[e] = cvt_bf16x2(bf16lo(m) + bf16lo(r[e]), bf16hi(m) + bf16hi(r[e]));
      else
        o4[e] = m;
    }
    *reinterpret_cast<uint4*>(yr + i) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
  };
  if constexpr (NCH > 0) {
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int i = c * 256 + lane * 8;
      if (i < width) emit(i, keep[c]);
    }
  } else {
    for (int i = lane * 8; i < width; i += 256) emit(i, *reinterpret_cast<const uint4*>(xr + i));
  }
}

// ------------------------------------------------------------------ RoPE
// In place on the Q and K columns of the fused QKV rows, with the rounding
// points of rotate_head in bf16 mode (packages/kernels/root.zig:615-633).
// One thread per (token, head, pair index).
__global__ void __launch_bounds__(256) rope_bf16_kernel(uint16_t* __restrict__ qkv, long long stride, int T,
                                                        int heads_qk, const float* __restrict__ cos_t,
                                                        const float* __restrict__ sin_t) {
  constexpr int HD = 64, HALF = 32;
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total = static_cast<long long>(T) * heads_qk * HALF;
  if (idx >= total) return;
  const int i = static_cast<int>(idx % HALF);
  const long long th = idx / HALF;
  const int head = static_cast<int>(th % heads_qk);
  const int t = static_cast<int>(th / heads_qk);
  uint16_t* v = qkv + t * stride + head * HD;
  const float* c = cos_t + static_cast<size_t>(t) * HD;
  const float* s = sin_t + static_cast<size_t>(t) * HD;
  auto rb = [](float f) { return bf16_to_f32(f32_to_bf16(f)); };
  const float first = bf16_to_f32(v[i]);
  const float second = bf16_to_f32(v[i + HALF]);
  const float cos_first = rb(c[i]), sin_first = rb(s[i]);
  const float cos_second = rb(c[i + HALF]), sin_second = rb(s[i + HALF]);
  const float left = rb(first * cos_first);
  const float right = rb(-second * sin_first);
  const float right2 = rb(first * sin_second);
  const float left2 = rb(second * cos_second);
  v[i] = f32_to_bf16(left + right);
  v[i + HALF] = f32_to_bf16(left2 + right2);
}

// ------------------------------------------------------ QK-norm + RoPE
// attention_impl with query/key norm weights (packages/kernels/root.zig:
// 500-530, bf16 mode): each Q head gets rms_norm_bf16 with q_norm, each K head
// with k_norm (root.zig:243-252), then rotate_head (:615-633), in place on the
// fused QKV rows. Eight threads per (token, head); thread j holds elements
// 8j..8j+7 of the 64-wide head.
//
// The sum of squares keeps the reference's order for 64 elements
// (pinned_torch_sum_squares_f32, root.zig:152-224: two 4x8 accumulator rows,
// no full level step): acc[r][l] = x[8r+l]^2 + x[8(r+4)+l]^2 for r < 4,
// vs[l] = ((acc[0][l] + acc[1][l]) + acc[2][l]) + acc[3][l], then
// sum = vs[0] + vs[1] + ... + vs[7]; every product and sum rounded on its own.
// The shuffles below reproduce exactly that, so the norm is bit-identical.
__global__ void __launch_bounds__(256) qk_norm_rope_bf16_kernel(uint16_t* __restrict__ qkv, long long stride, int T,
                                                                int heads, int kv_heads,
                                                                const uint16_t* __restrict__ q_norm,
                                                                const uint16_t* __restrict__ k_norm, float eps,
                                                                const float* __restrict__ cos_t,
                                                                const float* __restrict__ sin_t) {
  pdl_wait();
  pdl_launch_dependents();
  const int heads_qk = heads + kv_heads;
  const long long group = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 3;
  const int j = threadIdx.x & 7;
  // whole 8-lane groups drop out together, so the group's shuffles stay convergent
  if (group >= static_cast<long long>(T) * heads_qk) return;
  const unsigned gmask = 0xffu << (threadIdx.x & 24);
  const int head = static_cast<int>(group % heads_qk);
  const int t = static_cast<int>(group / heads_qk);
  uint16_t* hp = qkv + t * stride + head * 64 + j * 8;
  const uint4 raw = *reinterpret_cast<const uint4*>(hp);
  const uint32_t p[4] = {raw.x, raw.y, raw.z, raw.w};
  float v[8];
#pragma unroll
  for (int e = 0; e < 4; ++e) v[2 * e] = bf16lo(p[e]), v[2 * e + 1] = bf16hi(p[e]);
  const uint16_t* scale = head < heads ? q_norm : k_norm;
  if (scale != nullptr) {
    float acc[8];
#pragma unroll
    for (int l = 0; l < 8; ++l) {
      const float sq = __fmul_rn(v[l], v[l]);
      acc[l] = __fadd_rn(sq, __shfl_down_sync(gmask, sq, 4, 8));    // rows r and r+4 (valid in j < 4)
    }
    float sum = 0.f;
#pragma unroll
    for (int l = 0; l < 8; ++l) {
      float vs = __shfl_sync(gmask, acc[l], 0, 8);
      vs = __fadd_rn(vs, __shfl_sync(gmask, acc[l], 1, 8));
      vs = __fadd_rn(vs, __shfl_sync(gmask, acc[l], 2, 8));
      vs = __fadd_rn(vs, __shfl_sync(gmask, acc[l], 3, 8));
      sum = __fadd_rn(sum, vs);
    }
    const float inv = 1.0f / sqrtf(__fdiv_rn(sum, 64.f) + eps);
    const uint4 wv = __ldg(reinterpret_cast<const uint4*>(scale + j * 8));
    const uint32_t q[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint32_t n = cvt_bf16x2(__fmul_rn(v[2 * e], inv), __fmul_rn(v[2 * e + 1], inv));
      const uint32_t m = cvt_bf16x2(__fmul_rn(bf16lo(n), bf16lo(q[e])), __fmul_rn(bf16hi(n), bf16hi(q[e])));
      v[2 * e] = bf16lo(m), v[2 * e + 1] = bf16hi(m);
    }
  }
  uint32_t o4[4];
  if (cos_t != nullptr) {
    // pair (i, i+32): threads j and j^4 exchange their eight values
    const bool first_half = j < 4;
    const int col = j * 8;
    const float* c = cos_t + static_cast<size_t>(t) * 64;
    const float* s = sin_t + static_cast<size_t>(t) * 64;
    auto rb = [](float f) { return bf16_to_f32(f32_to_bf16(f)); };
    float r[8];
#pragma unroll
    for (int l = 0; l < 8; ++l) {
      const float other = __shfl_xor_sync(gmask, v[l], 4, 8);
      if (first_half) {
        // element i = col + l: left + right with first = own, second = partner
        const float left = rb(__fmul_rn(v[l], rb(c[col + l])));
        const float right = rb(__fmul_rn(-other, rb(s[col + l])));
        r[l] = __fadd_rn(left, right);
      } else {
        // element i + 32 = col + l: first = partner, second = own
        const float left2 = rb(__fmul_rn(v[l], rb(c[col + l])));
        const float right2 = rb(__fmul_rn(other, rb(s[col + l])));
        r[l] = __fadd_rn(left2, right2);
      }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) o4[e] = cvt_bf16x2(r[2 * e], r[2 * e + 1]);
  } else {
#pragma unroll
    for (int e = 0; e < 4; ++e) o4[e] = cvt_bf16x2(v[2 * e], v[2 * e + 1]);
  }
  *reinterpret_cast<uint4*>(hp) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
}

// --------------------------------------------------------- V transpose
// vt[(kvh*64 + d) * T + t] = qkv[t * stride + voff + kvh*64 + d], 64x64 tiles.
__global__ void __launch_bounds__(256) v_transpose_kernel(const uint16_t* __restrict__ qkv, long long stride,
                                                          long long voff, int T, int vwidth,
                                                          uint16_t* __restrict__ vt) {
  __shared__ uint16_t tile[64][66];
  const int t0 = blockIdx.x * 64, c0 = blockIdx.y * 64;
  const int tx = threadIdx.x & 63, ty = threadIdx.x >> 6;  // 64 x 4
  for (int r = ty; r < 64; r += 4) {
    const int t = t0 + r, c = c0 + tx;
    tile[r][tx] = (t < T && c < vwidth) ? qkv[t * stride + voff + c] : uint16_t(0);
  }
  __syncthreads();
  for (int r = ty; r < 64; r += 4) {
    const int c = c0 + r, t = t0 + tx;
    if (c < vwidth && t < T) vt[static_cast<size_t>(c) * T + t] = tile[tx][r];
  }
}

// --------------------------------------------------------------- SwiGLU
// out[t, i] = bf16(bf16(g / (1 + exp(-g))) * u), g = gate_up[t, i], u = gate_up[t, F + i]
// (silu_bf16 root.zig:264-269 and the product at decoder.zig:210).
__global__ void __launch_bounds__(256) silu_mul_bf16_kernel(const uint16_t* __restrict__ gu,
                                                            uint16_t* __restrict__ out, int T, int F) {
  const long long idx = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  if (idx >= static_cast<long long>(T) * F) return;
  const int t = static_cast<int>(idx / F);
  const int i = static_cast<int>(idx % F);
  const uint4 g = *reinterpret_cast<const uint4*>(gu + static_cast<size_t>(t) * 2 * F + i);
  const uint4 u = *reinterpret_cast<const uint4*>(gu + static_cast<size_t>(t) * 2 * F + F + i);
  const uint32_t gp[4] = {g.x, g.y, g.z, g.w}, up[4] = {u.x, u.y, u.z, u.w};
  uint32_t o4[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float g0 = bf16lo(gp[e]), g1 = bf16hi(gp[e]);
    const float s0 = bf16_to_f32(f32_to_bf16(g0 / (1.0f + expf(-g0))));
    const float s1 = bf16_to_f32(f32_to_bf16(g1 / (1.0f + expf(-g1))));
    o4[e] = pack_bf16x2(s0 * bf16lo(up[e]), s1 * bf16hi(up[e]));
  }
  *reinterpret_cast<uint4*>(out + idx) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
}

// h = bf16(h + a) (decoder.zig:310-313), 8 elements per thread
__global__ void __launch_bounds__(256) add_bf16_kernel(uint16_t* __restrict__ h, const uint16_t* __restrict__ a,
                                                       long long n) {
  const long long idx = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  if (idx >= n) return;
  const uint4 x = *reinterpret_cast<const uint4*>(h + idx);
  const uint4 y = *reinterpret_cast<const uint4*>(a + idx);
  const uint32_t xp[4] = {x.x, x.y, x.z, x.w}, yp[4] = {y.x, y.y, y.z, y.w};
  uint32_t o4[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) o4[e] = pack_bf16x2(bf16lo(xp[e]) + bf16lo(yp[e]), bf16hi(xp[e]) + bf16hi(yp[e]));
  *reinterpret_cast<uint4*>(h + idx) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
}

// h[t] = bf16(h[t] + level_embedding[level(t)]) for target rows (ncm_model.zig:159-168)
__global__ void __launch_bounds__(256) add_level_embedding_kernel(uint16_t* __restrict__ h,
                                                                  const uint16_t* __restrict__ emb,
                                                                  const int* __restrict__ row_level, int T,
                                                                  int width) {
  const long long idx = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  if (idx >= static_cast<long long>(T) * width) return;
  const int t = static_cast<int>(idx / width);
  const int c = static_cast<int>(idx % width);
  const int lv = row_level[t];
  if (lv < 0) return;
  const uint4 x = *reinterpret_cast<const uint4*>(h + idx);
  const uint4 y = __ldg(reinterpret_cast<const uint4*>(emb + static_cast<size_t>(lv) * width + c));
  const uint32_t xp[4] = {x.x, x.y, x.z, x.w}, yp[4] = {y.x, y.y, y.z, y.w};
  uint32_t o4[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) o4[e] = pack_bf16x2(bf16lo(xp[e]) + bf16lo(yp[e]), bf16hi(xp[e]) + bf16hi(yp[e]));
  *reinterpret_cast<uint4*>(h + idx) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
}

// out[t] = table[ids[t]] (embedding_row, root.zig:288-301); bad ids raise the error word
__global__ void __launch_bounds__(256) embedding_gather_kernel(const uint16_t* __restrict__ table, int vocab,
                                                               int width, const int32_t* __restrict__ ids, int T,
                                                               uint16_t* __restrict__ out, int* err) {
  const int t = blockIdx.x;
  if (t >= T) return;
  const int id = ids[t];
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) atomicOr(err, kErrBadIndex);
    return;
  }
  const uint4* src = reinterpret_cast<const uint4*>(table + static_cast<size_t>(id) * width);
  uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(t) * width);
  for (int i = threadIdx.x; i < width / 8; i += blockDim.x) dst[i] = __ldg(src + i);
}

inline unsigned blocks_for(long long n, long long per_block) { return static_cast<unsigned>((n + per_block - 1) / per_block); }

}  // namespace

cudaError_t launch_rms_norm_bf16(const uint16_t* x, const uint16_t* w, const uint16_t* b, uint16_t* y, int rows,
                                 int width, float eps, cudaStream_t st) {
  const int blocks = (rows + 7) / 8;
  if (width <= 1024)
    return launch_pdl(rms_norm_bf16_kernel<4>, dim3(blocks), dim3(256), 0, st, 1, x, w, b, y, rows, width, eps);
  else if (width <= 2048)
    return launch_pdl(rms_norm_bf16_kernel<8>, dim3(blocks), dim3(256), 0, st, 1, x, w, b, y, rows, width, eps);
  else if (width <= 4096)
    return launch_pdl(rms_norm_bf16_kernel<16>, dim3(blocks), dim3(256), 0, st, 1, x, w, b, y, rows, width, eps);
  else
    return launch_pdl(rms_norm_bf16_kernel<0>, dim3(blocks), dim3(256), 0, st, 1, x, w, b, y, rows, width, eps);
}

cudaError_t launch_rope_bf16(uint16_t* qkv, long long stride, int T, int heads_qk, const float* c, const float* s,
                             cudaStream_t st) {
  rope_bf16_kernel<<<blocks_for(static_cast<long long>(T) * heads_qk * 32, 256), 256, 0, st>>>(qkv, stride, T,
                                                                                             heads_qk, c, s);
  return cudaGetLastError();
}

cudaError_t launch_qk_norm_rope_bf16(uint16_t* qkv, long long stride, int T, int heads, int kv_heads,
                                     const uint16_t* q_norm, const uint16_t* k_norm, float eps, const float* c,
                                     const float* s, cudaStream_t st) {
  const long long threads = static_cast<long long>(T) * (heads + kv_heads) * 8;
  return launch_pdl(qk_norm_rope_bf16_kernel, dim3(blocks_for(threads, 256)), dim3(256), 0, st, 1, qkv, stride, T,
                    heads, kv_heads, q_norm, k_norm, eps, c, s);
}

cudaError_t launch_v_transpose(const uint16_t* qkv, long long stride, long long voff, int T, int vwidth, uint16_t* vt,
                               cudaStream_t st) {
  dim3 grid(blocks_for(T, 64), blocks_for(vwidth, 64));
  v_transpose_kernel<<<grid, 256, 0, st>>>(qkv, stride, voff, T, vwidth, vt);
  return cudaGetLastError();
}

cudaError_t launch_silu_mul_bf16(const uint16_t* gu, uint16_t* out, int T, int F, cudaStream_t st) {
  silu_mul_bf16_kernel<<<blocks_for(static_cast<long long>(T) * F / 8, 256), 256, 0, st>>>(gu, out, T, F);
  return cudaGetLastError();
}

cudaError_t launch_add_bf16(uint16_t* h, const uint16_t* a, long long n, cudaStream_t st) {
  add_bf16_kernel<<<blocks_for(n / 8, 256), 256, 0, st>>>(h, a, n);
  return cudaGetLastError();
}

cudaError_t launch_add_level_embedding(uint16_t* h, const uint16_t* emb, const int* row_level, int T, int width,
                                       cudaStream_t st) {
  add_level_embedding_kernel<<<blocks_for(static_cast<long long>(T) * width / 8, 256), 256, 0, st>>>(
      h, emb, row_level, T, width);
  return cudaGetLastError();
}

cudaError_t launch_embedding_gather(const uint16_t* table, int vocab, int width, const int32_t* ids, int T,
                                    uint16_t* out, int* err, cudaStream_t st) {
  embedding_gather_kernel<<<T, 128, 0, st>>>(table, vocab, width, ids, T, out, err);
  return cudaGetLastError();
}

// RoPE inverse frequencies with libm, in the reference's f32 operation order:
// rope_default (packages/kernels/root.zig:305-316, :668-674), and with
// `llama3` the Llama 3 adjustment of rope_llama3 (root.zig:636-666).
void rope_inv_freq(int head_dim, float theta, const RopeLlama3* llama3, float* inv) {
  const int half = head_dim / 2;
  const float hdf = static_cast<float>(head_dim);
  for (int i = 0; i < half; ++i) inv[i] = 1.0f / powf(theta, static_cast<float>(2 * i) / hdf);
  if (llama3 == nullptr) return;
  const float factor = llama3->factor, low = llama3->low_freq_factor, high = llama3->high_freq_factor;
  const float old_ctx = static_cast<float>(llama3->original_max_position_embeddings);
  const float low_wl =
      static_cast<float>(static_cast<double>(llama3->original_max_position_embeddings) / static_cast<double>(low));
  const float high_wl =
      static_cast<float>(static_cast<double>(llama3->original_max_position_embeddings) / static_cast<double>(high));
  const float two_pi = static_cast<float>(2.0 * 3.14159265358979323846);
  for (int i = 0; i < half; ++i) {
    const float f = inv[i];
    const float wl = two_pi / f;
    const float lf = wl > low_wl ? f / factor : f;
    const float sm = (old_ctx / wl - low) / (high - low);
    const float smoothed = (1.0f - sm) * lf / factor + sm * lf;
    const bool medium = !(wl < high_wl) && !(wl > low_wl);
    inv[i] = medium ? smoothed : lf;
  }
}

// RoPE cos/sin tables at explicit positions, on the host with libm exactly as
// rope_tables + tables_at_positions compute them (packages/kernels/root.zig:318-348,
// src/ncm_position.zig:71-118), from rope_default's or rope_llama3's frequencies.
void rope_tables_host(int head_dim, float theta, const int* positions, int T, float* cos_out, float* sin_out,
                      const RopeLlama3* llama3) {
  const int half = head_dim / 2;
  std::vector<float> inv(half);
  rope_inv_freq(head_dim, theta, llama3, inv.data());
  for (int t = 0; t < T; ++t) {
    const float pf = static_cast<float>(positions[t]);
    for (int i = 0; i < half; ++i) {
      const float ang = pf * inv[i];
      const float cv = cosf(ang), sv = sinf(ang);
      cos_out[t * head_dim + i] = cv;
      cos_out[t * head_dim + half + i] = cv;
      sin_out[t * head_dim + i] = sv;
      sin_out[t * head_dim + half + i] = sv;
    }
  }
}

}  // namespace ncm
