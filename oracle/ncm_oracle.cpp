// CPU oracle for ncmorph_b200 — TEST INFRASTRUCTURE ONLY (see ncm_oracle.h).
//
// Compiled with -ffp-contract=off: products and sums are rounded separately
// exactly where the reference's strict-float Zig does, and fused only where
// the reference calls @mulAdd (written here as fmaf).
#include "ncm_oracle.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <vector>

#if defined(__AVX2__) || defined(__AVX512F__)
#include <immintrin.h>
#endif
#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

inline uint32_t f2u(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  return u;
}
inline float u2f(uint32_t u) {
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

// packages/bf16/root.zig:17-22 — RNE, every NaN -> 0x7FC0
inline uint16_t bf16_from(float v) {
  const uint32_t x = f2u(v);
  if ((x & 0x7FFFFFFFu) > 0x7F800000u) return 0x7FC0;
  const uint32_t bias = 0x7FFFu + ((x >> 16) & 1u);
  return static_cast<uint16_t>((x + bias) >> 16);
}
// packages/bf16/root.zig:25-27
inline float bf16_to(uint16_t b) { return u2f(static_cast<uint32_t>(b) << 16); }
// packages/kernels/root.zig:10-12
inline float rb(float v) { return bf16_to(bf16_from(v)); }
inline float mrb(float v, bool on) { return on ? rb(v) : v; }
// packages/kernels/root.zig:144-148
inline float ftz(float v) {
  const uint32_t b = f2u(v);
  if ((b & 0x7F800000u) == 0) return u2f(b & 0x80000000u);
  return v;
}

const float kInf = std::numeric_limits<float>::infinity();

// Lane-wise fused multiply-add for the RVQ distance loop: each lane is one
// independent fmaf chain, so the vector width changes speed, not results.
#if defined(__AVX512F__)
constexpr size_t kVecW = 16;
struct VecF {
  __m512 v;
};
inline VecF vzero() { return {_mm512_setzero_ps()}; }
inline VecF vload(const float* p) { return {_mm512_loadu_ps(p)}; }
inline VecF vfma_bcast(float a, VecF b, VecF c) { return {_mm512_fmadd_ps(_mm512_set1_ps(a), b.v, c.v)}; }
inline void vstore(float* p, VecF v) { _mm512_storeu_ps(p, v.v); }
#elif defined(__AVX2__) && defined(__FMA__)
constexpr size_t kVecW = 8;
struct VecF {
  __m256 v;
};
inline VecF vzero() { return {_mm256_setzero_ps()}; }
inline VecF vload(const float* p) { return {_mm256_loadu_ps(p)}; }
inline VecF vfma_bcast(float a, VecF b, VecF c) { return {_mm256_fmadd_ps(_mm256_set1_ps(a), b.v, c.v)}; }
inline void vstore(float* p, VecF v) { _mm256_storeu_ps(p, v.v); }
#else
constexpr size_t kVecW = 8;
struct VecF {
  float v[8];
};
inline VecF vzero() { return VecF{}; }
inline VecF vload(const float* p) {
  VecF r;
  for (size_t i = 0; i < 8; ++i) r.v[i] = p[i];
  return r;
}
inline VecF vfma_bcast(float a, VecF b, VecF c) {
  for (size_t i = 0; i < 8; ++i) c.v[i] = std::fmaf(a, b.v[i], c.v[i]);
  return c;
}
inline void vstore(float* p, VecF v) {
  for (size_t i = 0; i < 8; ++i) p[i] = v.v[i];
}
#endif

// packages/kernels/root.zig:106-142, one output element.
inline float matmul_bf16_elem(const float* x, const float* w, const float* bias, size_t o, size_t in_w) {
  const size_t rbs = std::min(in_w, in_w > 1024 ? size_t(1024) : size_t(512));
  float sum = 0.0f;
  for (size_t bs = 0; bs < in_w; bs += rbs) {
    const size_t be = std::min(bs + rbs, in_w);
    float partial = 0.0f;
    size_t i = bs;
    while (i + 1 < be) {
      const float xh = ftz(rb(x[i + 1]));
      const float wh = ftz(rb(w[i + 1]));
      const float xl = ftz(rb(x[i]));
      const float wl = ftz(rb(w[i]));
      partial = ftz(std::fmaf(xh, wh, partial));
      partial = ftz(std::fmaf(xl, wl, partial));
      i += 2;
    }
    if (i < be) partial = ftz(std::fmaf(ftz(rb(x[i])), ftz(rb(w[i])), partial));
    sum += partial;
  }
  if (bias != nullptr) sum += rb(bias[o]);
  return rb(sum);
}

// packages/kernels/root.zig:583-609 (project)
void project(const float* in, const float* w, const float* bias, float* out, size_t T, size_t in_w, size_t out_w,
             bool bf16_mode) {
  if (bf16_mode) {
    orc_matmul_bf16(in, w, bias, out, T, in_w, out_w);
    return;
  }
  orc_matmul(in, w, out, T, in_w, out_w);
  if (bias != nullptr)
    for (size_t t = 0; t < T; ++t)
      for (size_t o = 0; o < out_w; ++o) out[t * out_w + o] += bias[o];
}

// packages/kernels/root.zig:615-633
void rotate_head(float* v, const float* c, const float* s, size_t n, bool bm) {
  const size_t h = n / 2;
  for (size_t i = 0; i < h; ++i) {
    const float first = v[i];
    const float second = v[i + h];
    const float cos_first = mrb(c[i], bm);
    const float sin_first = mrb(s[i], bm);
    const float cos_second = mrb(c[i + h], bm);
    const float sin_second = mrb(s[i + h], bm);
    const float left = mrb(first * cos_first, bm);
    const float right = mrb(-second * sin_first, bm);
    const float right2 = mrb(first * sin_second, bm);
    const float left2 = mrb(second * cos_second, bm);
    v[i] = mrb(left + right, bm);
    v[i + h] = mrb(left2 + right2, bm);
  }
}

// packages/kernels/root.zig:537-575: one query row and head against every
// key row: bf16-mode scores bf16(bf16(q.k) * 1/sqrt(hd)) over the allowed
// keys, softmax, bf16 probabilities, context sums in increasing key order.
void attend_row(const float* q, const float* Kt, const float* V, size_t T, size_t kvw, size_t kvh, size_t hd,
                const uint8_t* mask_row, bool bm, float* sc, float* pr, float* c) {
  const float scale = 1.0f / std::sqrt(static_cast<float>(hd));
  bool any = false;
  for (size_t ki = 0; ki < T; ++ki) {
    if (!mask_row[ki]) {
      sc[ki] = -kInf;
      continue;
    }
    any = true;
    const float* k = &Kt[ki * kvw + kvh * hd];
    float s = 0.0f;
    for (size_t d = 0; d < hd; ++d) s += q[d] * k[d];
    const float sv = mrb(s, bm);
    sc[ki] = mrb(sv * scale, bm);
  }
  if (any) {
    orc_softmax(sc, pr, T);
    if (bm)
      for (size_t ki = 0; ki < T; ++ki) pr[ki] = rb(pr[ki]);
  } else {
    std::fill(pr, pr + T, 0.0f);
  }
  for (size_t d = 0; d < hd; ++d) {
    float s = 0.0f;
    for (size_t ki = 0; ki < T; ++ki) s += pr[ki] * V[ki * kvw + kvh * hd + d];
    c[d] = mrb(s, bm);
  }
}

}  // namespace

extern "C" {

uint16_t orc_bf16_from_f32(float v) { return bf16_from(v); }
float orc_bf16_to_f32(uint16_t b) { return bf16_to(b); }
void orc_bf16_from_f32_n(const float* x, uint16_t* y, size_t n) {
  for (size_t i = 0; i < n; ++i) y[i] = bf16_from(x[i]);
}
void orc_round_bf16_n(const float* x, float* y, size_t n) {
  for (size_t i = 0; i < n; ++i) y[i] = rb(x[i]);
}

// packages/kernels/root.zig:25-65: 32-wide tiles over tokens, outputs and
// inputs; each output accumulates in increasing k.
void orc_matmul(const float* in, const float* w, float* out, size_t T, size_t in_w, size_t out_w) {
  const size_t B = 32;
  for (size_t t0 = 0; t0 < T; t0 += B) {
    const size_t t1 = std::min(t0 + B, T);
    for (size_t o0 = 0; o0 < out_w; o0 += B) {
      const size_t o1 = std::min(o0 + B, out_w);
      for (size_t t = t0; t < t1; ++t)
        for (size_t o = o0; o < o1; ++o) out[t * out_w + o] = 0.0f;
      for (size_t i0 = 0; i0 < in_w; i0 += B) {
        const size_t i1 = std::min(i0 + B, in_w);
        for (size_t t = t0; t < t1; ++t)
          for (size_t o = o0; o < o1; ++o) {
            float acc = out[t * out_w + o];
            for (size_t i = i0; i < i1; ++i) acc += in[t * in_w + i] * w[o * in_w + i];
            out[t * out_w + o] = acc;
          }
      }
    }
  }
}

// packages/kernels/root.zig:71-93
void orc_matmul_reference(const float* in, const float* w, float* out, size_t T, size_t in_w, size_t out_w) {
  for (size_t t = 0; t < T; ++t)
    for (size_t o = 0; o < out_w; ++o) {
      float s = 0.0f;
      for (size_t i = 0; i < in_w; ++i) s += in[t * in_w + i] * w[o * in_w + i];
      out[t * out_w + o] = s;
    }
}

void orc_matmul_bf16(const float* in, const float* w, const float* bias, float* out, size_t T, size_t in_w,
                     size_t out_w) {
  for (size_t t = 0; t < T; ++t)
    for (size_t o = 0; o < out_w; ++o) out[t * out_w + o] = matmul_bf16_elem(in + t * in_w, w + o * in_w, bias, o, in_w);
}

void orc_matmul_bf16_mt(const float* in, const float* w, const float* bias, float* out, size_t T, size_t in_w,
                        size_t out_w, int threads) {
  const long long total = static_cast<long long>(T) * static_cast<long long>(out_w);
#pragma omp parallel for num_threads(threads) schedule(static)
  for (long long e = 0; e < total; ++e) {
    const size_t t = static_cast<size_t>(e) / out_w;
    const size_t o = static_cast<size_t>(e) % out_w;
    out[e] = matmul_bf16_elem(in + t * in_w, w + o * in_w, bias, o, in_w);
  }
}

// packages/kernels/root.zig:152-224 — PyTorch's 8-lane AVX2 cascade order.
float orc_sum_squares_pinned(const float* x, size_t n) {
  const size_t vw = 8;
  const size_t vc = n / vw;
  const size_t row_count = vc / 4;
  size_t log2_rows = 0, log2_limit = 1;
  while (log2_limit < row_count) {
    ++log2_rows;
    log2_limit *= 2;
  }
  const size_t level_power = std::max<size_t>(4, log2_rows / 4);
  const size_t level_step = size_t(1) << level_power;
  const size_t level_mask = level_step - 1;
  float acc[4][4][8];
  std::memset(acc, 0, sizeof(acc));
  size_t ri = 0;
  while (ri + level_step <= row_count) {
    for (size_t s = 0; s < level_step; ++s)
      for (size_t r = 0; r < 4; ++r) {
        const size_t vi = (ri + s) * 4 + r;
        for (size_t l = 0; l < vw; ++l) {
          const float v = x[vi * vw + l];
          acc[0][r][l] += v * v;
        }
      }
    ri += level_step;
    for (size_t lv = 1; lv < 4; ++lv) {
      for (size_t r = 0; r < 4; ++r)
        for (size_t l = 0; l < vw; ++l) {
          acc[lv][r][l] += acc[lv - 1][r][l];
          acc[lv - 1][r][l] = 0.0f;
        }
      if ((ri & (level_mask << (lv * level_power))) != 0) break;
    }
  }
  for (size_t g = ri; g < row_count; ++g)
    for (size_t r = 0; r < 4; ++r) {
      const size_t vi = g * 4 + r;
      for (size_t l = 0; l < vw; ++l) {
        const float v = x[vi * vw + l];
        acc[0][r][l] += v * v;
      }
    }
  for (size_t lv = 1; lv < 4; ++lv)
    for (size_t r = 0; r < 4; ++r)
      for (size_t l = 0; l < vw; ++l) acc[0][r][l] += acc[lv][r][l];
  for (size_t vi = row_count * 4; vi < vc; ++vi)
    for (size_t l = 0; l < vw; ++l) {
      const float v = x[vi * vw + l];
      acc[0][0][l] += v * v;
    }
  float vs[8];
  for (size_t l = 0; l < vw; ++l) vs[l] = acc[0][0][l];
  for (size_t r = 1; r < 4; ++r)
    for (size_t l = 0; l < vw; ++l) vs[l] += acc[0][r][l];
  float sum = 0.0f;
  for (size_t i = vc * vw; i < n; ++i) sum += x[i] * x[i];
  for (size_t l = 0; l < vw; ++l) sum += vs[l];
  return sum;
}

// packages/kernels/root.zig:226-239
void orc_rms_norm(const float* in, const float* w, float* out, size_t n, float eps) {
  const float ss = orc_sum_squares_pinned(in, n);
  const float ms = ss / static_cast<float>(n);
  const float inv = 1.0f / std::sqrt(ms + eps);
  for (size_t i = 0; i < n; ++i) {
    const float nv = in[i] * inv;
    out[i] = nv * w[i];
  }
}

// packages/kernels/root.zig:243-252
void orc_rms_norm_bf16(const float* in, const float* w, float* out, size_t n, float eps) {
  const float ss = orc_sum_squares_pinned(in, n);
  const float ms = ss / static_cast<float>(n);
  const float inv = 1.0f / std::sqrt(ms + eps);
  for (size_t i = 0; i < n; ++i) {
    const float nv = rb(in[i] * inv);
    out[i] = rb(nv * rb(w[i]));
  }
}

// packages/kernels/root.zig:255-261 (std.math.exp restated as C expf)
void orc_silu(const float* in, float* out, size_t n) {
  for (size_t i = 0; i < n; ++i) {
    const float v = in[i];
    const float sg = 1.0f / (1.0f + std::exp(-v));
    out[i] = v * sg;
  }
}

// packages/kernels/root.zig:264-269
void orc_silu_bf16(const float* in, float* out, size_t n) {
  for (size_t i = 0; i < n; ++i) {
    const float v = in[i];
    out[i] = rb(v / (1.0f + std::exp(-v)));
  }
}

// packages/kernels/root.zig:272-285
void orc_softmax(const float* in, float* out, size_t n) {
  float m = in[0];
  for (size_t i = 1; i < n; ++i) m = std::max(m, in[i]);
  float s = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    out[i] = std::exp(in[i] - m);
    s += out[i];
  }
  for (size_t i = 0; i < n; ++i) out[i] /= s;
}

// src/ncm_norm.zig:21-49
void orc_rms_norm_rows(const float* in, const float* w, const float* bias, float* out, size_t rows, size_t width,
                       float eps) {
  for (size_t r = 0; r < rows; ++r) {
    orc_rms_norm(in + r * width, w, out + r * width, width, eps);
    if (bias != nullptr)
      for (size_t i = 0; i < width; ++i) out[r * width + i] += bias[i];
  }
}

// packages/kernels/root.zig:305-348, :668-674 (libm powf/cosf/sinf as the reference links them)
void orc_rope_default(size_t hd, float theta, size_t positions, float* inv_freq, float* cos_t, float* sin_t) {
  const float hdf = static_cast<float>(hd);
  for (size_t i = 0; i < hd / 2; ++i) {
    const float ex = static_cast<float>(2 * i) / hdf;
    inv_freq[i] = 1.0f / powf(theta, ex);
  }
  orc_rope_tables(inv_freq, hd / 2, positions, cos_t, sin_t);
}

void orc_rope_tables(const float* inv_freq, size_t half, size_t positions, float* cos_t, float* sin_t) {
  const size_t hd = half * 2;
  for (size_t p = 0; p < positions; ++p) {
    const float pf = static_cast<float>(p);
    for (size_t i = 0; i < half; ++i) {
      const float ang = pf * inv_freq[i];
      const float cv = cosf(ang), sv = sinf(ang);
      cos_t[p * hd + i] = cv;
      cos_t[p * hd + half + i] = cv;
      sin_t[p * hd + i] = sv;
      sin_t[p * hd + half + i] = sv;
    }
  }
}

// packages/kernels/root.zig:636-666
void orc_rope_llama3(size_t hd, float theta, float factor, float low_ff, float high_ff, size_t orig_max,
                     float* inv_freq) {
  const float hdf = static_cast<float>(hd);
  for (size_t i = 0; i < hd / 2; ++i) {
    const float ex = static_cast<float>(2 * i) / hdf;
    inv_freq[i] = 1.0f / powf(theta, ex);
  }
  const float old_ctx = static_cast<float>(orig_max);
  const float low_wl = static_cast<float>(static_cast<double>(orig_max) / static_cast<double>(low_ff));
  const float high_wl = static_cast<float>(static_cast<double>(orig_max) / static_cast<double>(high_ff));
  const float two_pi = static_cast<float>(2.0 * 3.14159265358979323846);
  for (size_t i = 0; i < hd / 2; ++i) {
    const float f = inv_freq[i];
    const float wl = two_pi / f;
    const float lf = wl > low_wl ? f / factor : f;
    const float sm = (old_ctx / wl - low_ff) / (high_ff - low_ff);
    const float smoothed = (1.0f - sm) * lf / factor + sm * lf;
    const bool medium = !(wl < high_wl) && !(wl > low_wl);
    inv_freq[i] = medium ? smoothed : lf;
  }
}

// packages/kernels/root.zig:380-399
void orc_causal_mask(const size_t* qpos, size_t nq, const size_t* kpos, size_t nk, long window, uint8_t* out) {
  for (size_t q = 0; q < nq; ++q)
    for (size_t k = 0; k < nk; ++k) {
      const bool causal = kpos[k] <= qpos[q];
      bool in_window = true;
      if (window > 0) {
        const size_t w = static_cast<size_t>(window);
        in_window = qpos[q] < w || kpos[k] > qpos[q] - w;
      }
      out[q * nk + k] = (causal && in_window) ? 1 : 0;
    }
}

static bool padded(const uint8_t* pm, size_t pl, size_t i) { return pl != 0 && pm[i] != 0; }

// src/ncm_mask.zig:10-42
int orc_block_diagonal_mask(size_t prefix, const size_t* levels, size_t nl, const uint8_t* pm, size_t pl,
                            uint8_t* out, size_t out_len) {
  if (pl != 0 && pl != prefix) return -1;
  size_t tgt = 0;
  for (size_t i = 0; i < nl; ++i) tgt += levels[i];
  const size_t S = prefix + tgt;
  if (out_len != S * S) return -2;
  std::memset(out, 0, out_len);
  for (size_t q = 0; q < prefix; ++q)
    for (size_t k = 0; k < prefix; ++k) out[q * S + k] = !padded(pm, pl, k);
  size_t off = prefix;
  for (size_t i = 0; i < nl; ++i) {
    for (size_t q = off; q < off + levels[i]; ++q) {
      for (size_t k = 0; k < prefix; ++k) out[q * S + k] = !padded(pm, pl, k);
      for (size_t k = off; k < off + levels[i]; ++k) out[q * S + k] = 1;
    }
    off += levels[i];
  }
  return 0;
}

// Block-causal over scales: the block-diagonal mask plus, for each level,
// every position of the earlier (coarser) levels. Not in ncmorph (its
// PROJECT.md D8 keeps block_causal out of scope); restated for the config
// whose mask is block-causal.
int orc_block_causal_mask(size_t prefix, const size_t* levels, size_t nl, const uint8_t* pm, size_t pl, uint8_t* out,
                          size_t out_len) {
  const int rc = orc_block_diagonal_mask(prefix, levels, nl, pm, pl, out, out_len);
  if (rc != 0) return rc;
  size_t tgt = 0;
  for (size_t i = 0; i < nl; ++i) tgt += levels[i];
  const size_t S = prefix + tgt;
  size_t off = prefix;
  for (size_t i = 0; i < nl; ++i) {
    for (size_t q = off; q < off + levels[i]; ++q)
      for (size_t k = prefix; k < off; ++k) out[q * S + k] = 1;
    off += levels[i];
  }
  return 0;
}

// src/ncm_position.zig:11-22
int orc_fill_level_positions(size_t prefix, const size_t* levels, size_t nl, size_t* out, size_t out_len) {
  size_t S = prefix;
  for (size_t i = 0; i < nl; ++i) S += levels[i];
  if (out_len != S) return -1;
  for (size_t p = 0; p < prefix; ++p) out[p] = p;
  size_t off = prefix;
  for (size_t i = 0; i < nl; ++i) {
    for (size_t p = 0; p < levels[i]; ++p) out[off + p] = p;
    off += levels[i];
  }
  return 0;
}

// src/ncm_model.zig:296-326: x <- x + conv1d_k3(x) (zero padding), weight [out][in][3]
int orc_apply_post_upsample_conv(float* x, const float* w, const float* b, size_t rows, size_t width) {
  std::vector<float> out(rows * width);
  for (size_t p = 0; p < rows; ++p)
    for (size_t oc = 0; oc < width; ++oc) {
      float v = b[oc];
      for (size_t ic = 0; ic < width; ++ic)
        for (size_t kk = 0; kk < 3; ++kk) {
          const long ip = static_cast<long>(p) + static_cast<long>(kk) - 1;
          if (ip < 0 || ip >= static_cast<long>(rows)) continue;
          v += w[oc * width * 3 + ic * 3 + kk] * x[static_cast<size_t>(ip) * width + ic];
        }
      out[p * width + oc] = x[p * width + oc] + v;
    }
  std::memcpy(x, out.data(), sizeof(float) * rows * width);
  return 0;
}

// packages/kernels/root.zig:450-581
int orc_attention(const float* in, const orc_attention_weights_t* W, size_t T, size_t hidden, size_t H, size_t Hkv,
                  size_t hd, float eps, const float* cos_t, const float* sin_t, const uint8_t* mask, float* out,
                  int bf16_mode, float* ctx_trace) {
  if (T == 0 || hidden == 0 || hd == 0 || H == 0 || Hkv == 0 || H % Hkv != 0) return -1;
  if ((W->q_norm == nullptr) != (W->k_norm == nullptr)) return -1;
  const bool bm = bf16_mode != 0;
  const size_t qw = H * hd, kvw = Hkv * hd;
  std::vector<float> Q(T * qw), Kt(T * kvw), V(T * kvw), C(T * qw);
  project(in, W->q_w, W->q_b, Q.data(), T, hidden, qw, bm);
  project(in, W->k_w, W->k_b, Kt.data(), T, hidden, kvw, bm);
  project(in, W->v_w, W->v_b, V.data(), T, hidden, kvw, bm);
  const size_t group = H / Hkv;
  for (size_t t = 0; t < T; ++t)
    for (size_t h = 0; h < H; ++h) {
      float* q = &Q[t * qw + h * hd];
      if (W->q_norm) {
        if (bm)
          orc_rms_norm_bf16(q, W->q_norm, q, hd, eps);
        else
          orc_rms_norm(q, W->q_norm, q, hd, eps);
      }
      rotate_head(q, cos_t + t * hd, sin_t + t * hd, hd, bm);
    }
  for (size_t t = 0; t < T; ++t)
    for (size_t h = 0; h < Hkv; ++h) {
      float* k = &Kt[t * kvw + h * hd];
      if (W->k_norm) {
        if (bm)
          orc_rms_norm_bf16(k, W->k_norm, k, hd, eps);
        else
          orc_rms_norm(k, W->k_norm, k, hd, eps);
      }
      rotate_head(k, cos_t + t * hd, sin_t + t * hd, hd, bm);
    }
  std::vector<float> sc(T), pr(T);
  for (size_t qi = 0; qi < T; ++qi)
    for (size_t h = 0; h < H; ++h)
      attend_row(&Q[qi * qw + h * hd], Kt.data(), V.data(), T, kvw, h / group, hd, mask + qi * T, bm, sc.data(),
                 pr.data(), &C[qi * qw + h * hd]);
  if (ctx_trace) std::memcpy(ctx_trace, C.data(), sizeof(float) * T * qw);
  project(C.data(), W->o_w, W->o_b, out, T, qw, hidden, bm);
  return 0;
}

// attention_impl's per-row core for a subset of query rows: Q [nrows, H*hd]
// (projected and rotated), K and V [T, Hkv*hd] (K rotated) of every row,
// mask rows [nrows, T]. Each output row is computed exactly as
// orc_attention computes that row; (row, head) pairs run in parallel.
int orc_attention_core_rows(const float* Q, const float* Kt, const float* V, const uint8_t* mask, size_t nrows,
                            size_t T, size_t H, size_t Hkv, size_t hd, float* ctx, int bf16_mode, int threads) {
  if (T == 0 || hd == 0 || H == 0 || Hkv == 0 || H % Hkv != 0) return -1;
  if (threads < 1) threads = 1;
  const bool bm = bf16_mode != 0;
  const size_t qw = H * hd, kvw = Hkv * hd, group = H / Hkv;
  const long long pairs = static_cast<long long>(nrows * H);
#pragma omp parallel num_threads(threads)
  {
    std::vector<float> sc(T), pr(T);
#pragma omp for schedule(dynamic, 4)
    for (long long e = 0; e < pairs; ++e) {
      const size_t r = static_cast<size_t>(e) / H, h = static_cast<size_t>(e) % H;
      attend_row(Q + r * qw + h * hd, Kt, V, T, kvw, h / group, hd, mask + r * T, bm, sc.data(), pr.data(),
                 ctx + r * qw + h * hd);
    }
  }
  return 0;
}

// rotate_head (packages/kernels/root.zig:615-633) over every head of n rows
// [n, heads*hd], row r with its own table row cos_t[r], sin_t[r] ([n, hd]).
void orc_rotate_rows(float* x, size_t n, size_t heads, size_t hd, const float* cos_t, const float* sin_t,
                     int bf16_mode) {
  for (size_t r = 0; r < n; ++r)
    for (size_t h = 0; h < heads; ++h) rotate_head(x + (r * heads + h) * hd, cos_t + r * hd, sin_t + r * hd, hd,
                                                   bf16_mode != 0);
}

// ------------------------------------------------------------------- RVQ
// ||e_k||^2: squares of bf16 values are exact in f64 and their f64 sum is
// exact for any realistic D; one rounding to f32.
void orc_code_sqnorm(const uint16_t* cb, float* out, size_t K, size_t D) {
  for (size_t k = 0; k < K; ++k) {
    double s = 0.0;
    for (size_t d = 0; d < D; ++d) {
      const double v = bf16_to(cb[k * D + d]);
      s += v * v;
    }
    out[k] = static_cast<float>(s);
  }
}

// One RVQ level (vq_forward_semantics.md:68-72, distance :81):
//   dist_k = fmaf(-2, dot_k, ||e_k||^2), dot_k = sequential fmaf over d of bf16(r)_d * e_kd
//   best = lowest k with the minimal dist (torch.argmin tie rule)
//   r -= e[code] (f32), code = codes_in[n] when teacher-forcing, else best.
// Work is split into (4-row block x code chunk) tasks; each output's dot
// product is the same sequential chain whatever the split, and chunk results
// merge in increasing code order, so threads change speed, not bits.
namespace {
struct Top2 {
  float best, second;
  int32_t idx;
};
}  // namespace

void orc_rvq_level(float* resid, const uint16_t* cb, const float* sqnorm, const int32_t* codes_in,
                   int32_t* best_out, float* rel_gap, size_t N, size_t D, size_t K, int threads) {
  constexpr size_t KB = kVecW;  // codes per block (one vector of independent accumulators)
  constexpr size_t RB = 8;      // rows per block
  if (threads < 1) threads = 1;
  const size_t Kp = (K + KB - 1) / KB * KB;
  std::vector<float> eT(D * Kp);  // codebook transposed to [D][Kp], zero-padded
#pragma omp parallel for num_threads(threads) schedule(static)
  for (long long d0 = 0; d0 < static_cast<long long>(D); d0 += 16) {
    const size_t d1 = std::min(static_cast<size_t>(d0) + 16, D);
    for (size_t k = 0; k < Kp; ++k)
      for (size_t d = static_cast<size_t>(d0); d < d1; ++d)
        eT[d * Kp + k] = k < K ? bf16_to(cb[k * D + d]) : 0.0f;
  }
  const size_t nblk = (N + RB - 1) / RB;
  const size_t kblocks = Kp / KB;
  size_t nchunk = 1;
  while (nblk * nchunk < static_cast<size_t>(threads) * 4 && nchunk * 2 <= kblocks) nchunk *= 2;
  const size_t kb_per_chunk = (kblocks + nchunk - 1) / nchunk;
  std::vector<float> a(nblk * RB * D);  // bf16(r), per block transposed to [d][RB]
  std::vector<double> a2(nblk * RB, 0.0);
#pragma omp parallel for num_threads(threads) schedule(static)
  for (long long n = 0; n < static_cast<long long>(nblk * RB); ++n) {
    const size_t blk = static_cast<size_t>(n) / RB, r = static_cast<size_t>(n) % RB;
    double s = 0.0;
    for (size_t d = 0; d < D; ++d) {
      const float v = static_cast<size_t>(n) < N ? rb(resid[n * D + d]) : 0.0f;
      a[(blk * D + d) * RB + r] = v;
      s += static_cast<double>(v) * v;
    }
    a2[n] = s;
  }
  std::vector<Top2> part(nblk * RB * nchunk);
  const long long tasks = static_cast<long long>(nblk * nchunk);
#pragma omp parallel for num_threads(threads) schedule(dynamic, 1)
  for (long long t = 0; t < tasks; ++t) {
    const size_t blk = static_cast<size_t>(t) / nchunk;
    const size_t ch = static_cast<size_t>(t) % nchunk;
    const size_t n0 = blk * RB;
    const size_t nr = std::min(RB, N - n0);
    Top2 tp[RB];
    for (size_t r = 0; r < RB; ++r) tp[r] = Top2{kInf, kInf, static_cast<int32_t>(ch * kb_per_chunk * KB)};
    const size_t kb0 = ch * kb_per_chunk, kb1 = std::min(kblocks, kb0 + kb_per_chunk);
    for (size_t kb = kb0; kb < kb1; ++kb) {
      const size_t k0 = kb * KB;
      VecF vacc[RB];
      for (size_t r = 0; r < RB; ++r) vacc[r] = vzero();
      const float* ab = &a[blk * D * RB];
      for (size_t d = 0; d < D; ++d) {
        const VecF e = vload(&eT[d * Kp + k0]);
        for (size_t r = 0; r < RB; ++r) vacc[r] = vfma_bcast(ab[d * RB + r], e, vacc[r]);
      }
      float acc[RB][KB];
      for (size_t r = 0; r < RB; ++r) vstore(acc[r], vacc[r]);
      for (size_t r = 0; r < nr; ++r)
        for (size_t j = 0; j < KB && k0 + j < K; ++j) {
          const float dist = std::fmaf(-2.0f, acc[r][j], sqnorm[k0 + j]);
          if (dist < tp[r].best) {
            tp[r].second = tp[r].best;
            tp[r].best = dist;
            tp[r].idx = static_cast<int32_t>(k0 + j);
          } else if (dist < tp[r].second) {
            tp[r].second = dist;
          }
        }
    }
    for (size_t r = 0; r < RB; ++r) part[(n0 + r) * nchunk + ch] = tp[r];
  }
#pragma omp parallel for num_threads(threads) schedule(static)
  for (long long nn = 0; nn < static_cast<long long>(N); ++nn) {
    const size_t n = static_cast<size_t>(nn);
    Top2 m = part[n * nchunk];
    for (size_t ch = 1; ch < nchunk; ++ch) {
      const Top2& c = part[n * nchunk + ch];
      if (c.best < m.best) {  // strict: on equal distances the lower code (earlier chunk) stays
        m.second = std::min(m.best, c.second);
        m.best = c.best;
        m.idx = c.idx;
      } else {
        m.second = std::min(m.second, c.best);
      }
    }
    if (best_out) best_out[n] = m.idx;
    if (rel_gap) {
      const double full = a2[n] + static_cast<double>(m.best);
      const double gap = static_cast<double>(m.second) - static_cast<double>(m.best);
      rel_gap[n] = static_cast<float>(gap / std::max(full, 1e-30));
    }
    const int32_t code = codes_in ? codes_in[n] : m.idx;
    if (code < 0 || static_cast<size_t>(code) >= K) continue;
    for (size_t d = 0; d < D; ++d) resid[n * D + d] -= bf16_to(cb[static_cast<size_t>(code) * D + d]);
  }
}

// vq_forward_semantics.md:69,82 — recon = sum over levels of the chosen codewords (f32, level order)
void orc_rvq_decode(const int32_t* codes, const uint16_t* cbs, size_t L, float* recon, size_t N, size_t D, size_t K) {
  for (size_t n = 0; n < N; ++n)
    for (size_t d = 0; d < D; ++d) {
      float acc = 0.0f;
      for (size_t l = 0; l < L; ++l) {
        const int32_t c = codes[l * N + n];
        acc += bf16_to(cbs[(l * K + static_cast<size_t>(c)) * D + d]);
      }
      recon[n * D + d] = acc;
    }
}

// vq_forward_semantics.md:67,80: F.interpolate(mode="area") with an integer
// factor = mean of f consecutive rows, summed in increasing order.
void orc_pool_avg(const float* x, float* y, size_t B, size_t T, size_t D, size_t f) {
  const size_t To = T / f;
  for (size_t b = 0; b < B; ++b)
    for (size_t j = 0; j < To; ++j)
      for (size_t d = 0; d < D; ++d) {
        const float* src = x + (b * T + j * f) * D + d;
        float s = src[0];
        for (size_t i = 1; i < f; ++i) s += src[i * D];
        y[(b * To + j) * D + d] = s / static_cast<float>(f);
      }
}

// Multiscale step: q = sum_l e_l[code] (f32, level order) per pooled row,
// nearest-repeat upsampled; r -= q, recon += q.
void orc_scale_update(const int32_t* codes, const uint16_t* cbs, size_t L, float* resid, float* recon, size_t B,
                      size_t T, size_t D, size_t K, size_t f) {
  const size_t P = B * (T / f);
  std::vector<float> q(D);
  for (size_t p = 0; p < P; ++p) {
    for (size_t d = 0; d < D; ++d) {
      float acc = 0.0f;
      for (size_t l = 0; l < L; ++l) acc += bf16_to(cbs[(l * K + static_cast<size_t>(codes[l * P + p])) * D + d]);
      q[d] = acc;
    }
    for (size_t i = 0; i < f; ++i) {
      const size_t row = p * f + i;
      for (size_t d = 0; d < D; ++d) {
        resid[row * D + d] -= q[d];
        recon[row * D + d] += q[d];
      }
    }
  }
}

// Upsampling along time as F.interpolate(size=T) on [B, C, T] data
// (research/reference/vq_forward_semantics.md:82, :108; PyTorch's
// upsample_linear1d / upsample_nearest1d CPU kernels), in their operation
// order: s = float(Tq) / float(T); nearest: i = min(floor(t * s), Tq - 1);
// linear: src = max(fma(s, t + 0.5, -0.5), 0), i0 = trunc(src),
// l1 = clamp(src - i0, 0, 1), out = fma(q[i0], 1 - l1, q[i1] * l1).
void orc_upsample(const float* q, float* out, size_t B, size_t Tq, size_t T, size_t D, int mode) {
  const float s = static_cast<float>(Tq) / static_cast<float>(T);
  for (size_t b = 0; b < B; ++b)
    for (size_t t = 0; t < T; ++t) {
      const float* qb = q + b * Tq * D;
      float* o = out + (b * T + t) * D;
      if (mode == 0) {
        size_t i0 = static_cast<size_t>(std::floor(static_cast<float>(t) * s));
        if (i0 > Tq - 1) i0 = Tq - 1;
        for (size_t d = 0; d < D; ++d) o[d] = qb[i0 * D + d];
      } else {
        float src = std::fma(s, static_cast<float>(t) + 0.5f, -0.5f);
        if (src < 0.f) src = 0.f;
        const size_t i0 = static_cast<size_t>(src);
        const float l1 = std::min(std::max(src - static_cast<float>(i0), 0.f), 1.f);
        const float l0 = 1.f - l1;
        const size_t i1 = i0 < Tq - 1 ? i0 + 1 : i0;
        for (size_t d = 0; d < D; ++d) {
          const float x1 = qb[i1 * D + d] * l1;
          o[d] = std::fma(qb[i0 * D + d], l0, x1);
        }
      }
    }
}

// Kernel-3 convolution with blend, per segment (zero padding at each
// segment's ends): out[t,o] = fma(alpha, x_blend[t,o], beta * (float(C) + b[o]))
// with C = sum_{i,k} w[o,i,k] * x_op[t+k-1,i] accumulated in f64 (the
// products of bf16 values are exact). Callers pass bf16-rounded x_op and w to
// mirror the tensor-core operands; apply_post_upsample_conv is alpha = beta = 1.
void orc_conv1d_k3(const float* x_op, const float* x_blend, const float* w, const float* b, float* out, size_t rows,
                   size_t width, const size_t* seg_lengths, size_t nseg, float alpha, float beta) {
  std::vector<size_t> seg_of(rows), seg_start(nseg ? nseg : 1), seg_end(nseg ? nseg : 1);
  if (seg_lengths == nullptr || nseg == 0) {
    seg_start[0] = 0, seg_end[0] = rows;
    for (size_t t = 0; t < rows; ++t) seg_of[t] = 0;
  } else {
    size_t at = 0;
    for (size_t s = 0; s < nseg; ++s) {
      seg_start[s] = at;
      for (size_t i = 0; i < seg_lengths[s]; ++i) seg_of[at + i] = s;
      at += seg_lengths[s];
      seg_end[s] = at;
    }
  }
  std::vector<float> res(rows * width);
#pragma omp parallel for schedule(static)
  for (long tt = 0; tt < static_cast<long>(rows); ++tt) {
    const size_t t = static_cast<size_t>(tt);
    const size_t s = seg_of[t];
    for (size_t o = 0; o < width; ++o) {
      double c = 0.0;
      for (int k = 0; k < 3; ++k) {
        const long src = static_cast<long>(t) + k - 1;
        if (src < static_cast<long>(seg_start[s]) || src >= static_cast<long>(seg_end[s])) continue;
        const float* xr = x_op + static_cast<size_t>(src) * width;
        const float* wr = w + o * width * 3 + k;
        for (size_t i = 0; i < width; ++i) c += static_cast<double>(wr[i * 3]) * static_cast<double>(xr[i]);
      }
      const float cb = static_cast<float>(c) + (b != nullptr ? b[o] : 0.f);
      res[t * width + o] = std::fma(alpha, x_blend != nullptr ? x_blend[t * width + o] : 0.f, beta * cb);
    }
  }
  std::memcpy(out, res.data(), sizeof(float) * rows * width);
}

// General multiscale step: q = sum_l e_l[code] per pooled row (f32, level
// order); Q = up(q) (mode 0 nearest, 1 linear); with Phi (phi_w non-null,
// [D, D, 3] bf16 values as f32) Q = fma(1 - r, Q, r * (C + b)) where C is the
// convolution of bf16(Q) within each batch item; resid -= Q; acc += Q.
void orc_scale_update_ex(const int32_t* codes, const uint16_t* cbs, size_t L, float* resid, float* acc, size_t B,
                         size_t T, size_t D, size_t K, size_t f, int mode, const float* phi_w, const float* phi_b,
                         float ratio) {
  const size_t Tq = T / f, P = B * Tq;
  std::vector<float> q(P * D), Q(B * T * D);
  for (size_t p = 0; p < P; ++p)
    for (size_t d = 0; d < D; ++d) {
      float a = 0.0f;
      for (size_t l = 0; l < L; ++l) a += bf16_to(cbs[(l * K + static_cast<size_t>(codes[l * P + p])) * D + d]);
      q[p * D + d] = a;
    }
  orc_upsample(q.data(), Q.data(), B, Tq, T, D, mode);
  if (phi_w != nullptr) {
    std::vector<float> Qb(Q.size());
    for (size_t i = 0; i < Q.size(); ++i) Qb[i] = bf16_to(bf16_from(Q[i]));
    std::vector<size_t> segs(B, T);
    orc_conv1d_k3(Qb.data(), Q.data(), phi_w, phi_b, Q.data(), B * T, D, segs.data(), B, 1.f - ratio, ratio);
  }
  for (size_t i = 0; i < B * T * D; ++i) {
    if (resid != nullptr) resid[i] -= Q[i];
    acc[i] += Q[i];
  }
}

// Codebook-tied head (_TiedCodebookHead, PROJECT.md:222), in the module's
// operation order: neg_d2 = (2 z.E^T - E_sq) / d_scale; logits = neg_d2 *
// exp(log_inv_T) + bias. d_scale = mean(E_sq) (f64 sum of the f32 norms);
// each dot product is an exact f64 sum of bf16 products rounded to f32.
// With codes/gap non-null also the argmax (lowest k on ties) and the top-2
// logit gap per row.
void orc_tied_head(const float* z, const uint16_t* cb, const float* esq_in, const float* bias, float log_inv_T,
                   float* logits, int32_t* codes, float* gap, size_t T, size_t d, size_t K) {
  std::vector<float> esq(K);
  if (esq_in != nullptr)
    std::memcpy(esq.data(), esq_in, sizeof(float) * K);
  else
    orc_code_sqnorm(cb, esq.data(), K, d);
  double tot = 0.0;
  for (size_t k = 0; k < K; ++k) tot += static_cast<double>(esq[k]);
  const float dsc = static_cast<float>(tot / static_cast<double>(K));
  const float e = std::exp(log_inv_T);
  std::vector<float> eb(K * d);
  for (size_t i = 0; i < K * d; ++i) eb[i] = bf16_to(cb[i]);
#pragma omp parallel for schedule(static)
  for (long tt = 0; tt < static_cast<long>(T); ++tt) {
    const size_t t = static_cast<size_t>(tt);
    float best = -std::numeric_limits<float>::infinity(), second = best;
    int32_t bi = 0;
    for (size_t k = 0; k < K; ++k) {
      double acc = 0.0;
      for (size_t i = 0; i < d; ++i) acc += static_cast<double>(z[t * d + i]) * static_cast<double>(eb[k * d + i]);
      const float a = static_cast<float>(acc);
      const float neg = (2.0f * a - esq[k]) / dsc;
      const float l = neg * e + (bias != nullptr ? bias[k] : 0.0f);
      if (logits != nullptr) logits[t * K + k] = l;
      if (l > best) {
        second = best;
        best = l;
        bi = static_cast<int32_t>(k);
      } else if (l > second) {
        second = l;
      }
    }
    if (codes != nullptr) codes[t] = bi;
    if (gap != nullptr) gap[t] = best - second;
  }
}

// Pre-quantisation GroupNorm, affine=False: x, y [B, T, C]; statistics per
// (sample, group) over T x C/G values in f64, biased variance.
void orc_group_norm(const float* x, float* y, size_t B, size_t T, size_t C, size_t G, float eps) {
  const size_t cg = C / G;
  for (size_t b = 0; b < B; ++b)
    for (size_t g = 0; g < G; ++g) {
      double s = 0.0, ss = 0.0;
      for (size_t t = 0; t < T; ++t)
        for (size_t c = 0; c < cg; ++c) {
          const double v = x[(b * T + t) * C + g * cg + c];
          s += v;
          ss += v * v;
        }
      const double n = static_cast<double>(T * cg);
      const double mean = s / n, var = std::max(ss / n - mean * mean, 0.0);
      const float m = static_cast<float>(mean), r = static_cast<float>(1.0 / std::sqrt(var + eps));
      for (size_t t = 0; t < T; ++t)
        for (size_t c = 0; c < cg; ++c) {
          const size_t o = (b * T + t) * C + g * cg + c;
          y[o] = (x[o] - m) * r;
        }
    }
}

// Conv1d(C, C, 4, stride 4) on x [B, L, C] (w [C, C, 4], b [C] or null) ->
// y [B, L/4, C]; f64 sums of the given (bf16-valued) operands, rounded to f32.
void orc_conv_down4(const float* x, const float* w, const float* b, float* y, size_t B, size_t L, size_t C) {
  const size_t Lo = L / 4;
  for (size_t bb = 0; bb < B; ++bb)
    for (size_t j = 0; j < Lo; ++j)
      for (size_t o = 0; o < C; ++o) {
        double acc = b != nullptr ? b[o] : 0.0;
        for (size_t t = 0; t < 4; ++t)
          for (size_t i = 0; i < C; ++i)
            acc += static_cast<double>(w[(o * C + i) * 4 + t]) * x[(bb * L + 4 * j + t) * C + i];
        y[(bb * Lo + j) * C + o] = static_cast<float>(acc);
      }
}

// ConvTranspose1d(C, C, 4, stride 4) on x [B, L, C] (w [C_in, C_out, 4]) -> y [B, 4L, C].
void orc_conv_up4(const float* x, const float* w, const float* b, float* y, size_t B, size_t L, size_t C) {
  for (size_t bb = 0; bb < B; ++bb)
    for (size_t j = 0; j < L; ++j)
      for (size_t t = 0; t < 4; ++t)
        for (size_t o = 0; o < C; ++o) {
          double acc = b != nullptr ? b[o] : 0.0;
          for (size_t i = 0; i < C; ++i)
            acc += static_cast<double>(w[(i * C + o) * 4 + t]) * x[(bb * L + j) * C + i];
          y[(bb * 4 * L + 4 * j + t) * C + o] = static_cast<float>(acc);
        }
}

// Codebook EMA of one level (models/quant.py:485-500 as restated in
// vq_forward_semantics.md:141-173): counts and row sums per code (rows in
// increasing order, f32), then the EMA update in f32 with the count total in f64.
void orc_ema(const float* u, const int32_t* codes, size_t N, size_t D, size_t K, float* ema_count, float* ema_sum,
             float* codebook, float decay, float eps, float* counts_out, float* sums_out) {
  std::vector<float> cnt(K, 0.f), sum(K * D, 0.f);
  for (size_t n = 0; n < N; ++n) {
    const size_t k = static_cast<size_t>(codes[n]);
    cnt[k] += 1.f;
    for (size_t d = 0; d < D; ++d) sum[k * D + d] += u[n * D + d];
  }
  double tot = 0.0;
  for (size_t k = 0; k < K; ++k) {
    ema_count[k] = decay * ema_count[k] + (1.f - decay) * cnt[k];
    tot += ema_count[k];
  }
  const float nt = static_cast<float>(tot);
  for (size_t k = 0; k < K; ++k) {
    const float nhat = (ema_count[k] + eps) / (nt + static_cast<float>(K) * eps) * nt;
    for (size_t d = 0; d < D; ++d) {
      const size_t i = k * D + d;
      ema_sum[i] = decay * ema_sum[i] + (1.f - decay) * sum[i];
      codebook[i] = ema_sum[i] / nhat;
    }
  }
  if (counts_out) std::memcpy(counts_out, cnt.data(), sizeof(float) * K);
  if (sums_out) std::memcpy(sums_out, sum.data(), sizeof(float) * K * D);
}

}  // extern "C"
