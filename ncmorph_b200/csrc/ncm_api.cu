// C-ABI entry points of the NCM decoder forward (config 4): RMSNorm,
// embedding gather, RoPE tables, attention, and the full layer stack.
#include <algorithm>
#include <cstring>
#include <vector>

#include "internal.h"

namespace {

bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int ctx_ok(ncm_ctx* ctx) {
  if (ctx == nullptr) return ncm_fail(NCM_EINVAL, "null context");
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev != ctx->device) {
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e != cudaSuccess) return ncm_set_cuda_error(e);
  }
  return NCM_OK;
}

int check_mask(const ncm_mask_t* m, int64_t T) {
  if (m == nullptr) return ncm_fail(NCM_EINVAL, "attention: null mask");
  if (m->mode < 0 || m->mode > 2) return ncm_fail(NCM_EINVAL, "attention: mask mode %d unknown", m->mode);
  if (m->sliding_window < 0 || (m->sliding_window > 0 && m->mode != 0))
    return ncm_fail(NCM_EINVAL, "attention: sliding_window %d (non-negative, causal mode only)", m->sliding_window);
  if (m->mode == 0) return NCM_OK;
  if (m->prefix_length < 0 || m->prefix_length > 64)
    return ncm_fail(NCM_EINVAL, "attention: prefix_length %d outside [0, 64]", m->prefix_length);
  if (m->num_levels <= 0 || m->num_levels > 32) return ncm_fail(NCM_EINVAL, "attention: num_levels out of range");
  int64_t s = m->prefix_length;
  for (int i = 0; i < m->num_levels; ++i) {
    if (m->level_lengths[i] <= 0) return ncm_fail(NCM_EINVAL, "attention: level %d is empty", i);
    s += m->level_lengths[i];
  }
  if (s != T) return ncm_fail(NCM_EINVAL, "attention: prefix + levels = %lld but T = %lld", (long long)s, (long long)T);
  return NCM_OK;
}

}  // namespace

using namespace ncm;

extern "C" {

int ncm_rms_norm_bf16(ncm_ctx_t* ctx, const uint16_t* x, const uint16_t* w, const uint16_t* bias, uint16_t* y,
                      int64_t rows, int64_t width, float eps, ncm_stream_t stream) {
  int rc = ctx_ok(ctx);
  if (rc) return rc;
  if (rows <= 0 || width <= 0 || width % 8 != 0 || rows > INT32_MAX || width > INT32_MAX || !x || !w || !y)
    return ncm_fail(NCM_EINVAL, "rms_norm: bad arguments (rows=%lld width=%lld; width %% 8 == 0)", (long long)rows,
                    (long long)width);
  if (!a16(x) || !a16(w) || !a16(y) || (bias && !a16(bias)))
    return ncm_fail(NCM_EINVAL, "rms_norm: buffers must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Launch _l(ctx, KID_DECODER_ELEMENTWISE, st);
  NCM_CUDA_TRY(launch_rms_norm_bf16(x, w, bias, y, static_cast<int>(rows), static_cast<int>(width), eps, st));
  return NCM_OK;
}

int ncm_embedding_gather(ncm_ctx_t* ctx, const uint16_t* table, int64_t vocab, int64_t width, const int32_t* ids,
                         int64_t T, uint16_t* out, ncm_stream_t stream) {
  int rc = ctx_ok(ctx);
  if (rc) return rc;
  if (vocab <= 0 || width <= 0 || width % 8 != 0 || T <= 0 || T > INT32_MAX || vocab > INT32_MAX || !table || !ids ||
      !out)
    return ncm_fail(NCM_EINVAL, "embedding_gather: bad arguments");
  if (!a16(table) || !a16(out)) return ncm_fail(NCM_EINVAL, "embedding_gather: buffers must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Launch _l(ctx, KID_DECODER_ELEMENTWISE, st);
  NCM_CUDA_TRY(launch_embedding_gather(table, static_cast<int>(vocab), static_cast<int>(width), ids,
                                       static_cast<int>(T), out, ctx->d_err, st));
  return NCM_OK;
}

int ncm_rope_tables_host(int32_t head_dim, float theta, const int32_t* positions, int64_t T, float* cos_out,
                         float* sin_out) {
  if (head_dim <= 0 || head_dim % 2 != 0 || !(theta > 0.f) || T < 0 || (T > 0 && (!positions || !cos_out || !sin_out)))
    return ncm_fail(NCM_EINVAL, "rope_tables: bad arguments");
  rope_tables_host(head_dim, theta, positions, static_cast<int>(T), cos_out, sin_out);
  return NCM_OK;
}

int ncm_rope_tables_llama3_host(int32_t head_dim, float theta, float factor, float low_freq_factor,
                                float high_freq_factor, int64_t original_max_position_embeddings,
                                const int32_t* positions, int64_t T, float* cos_out, float* sin_out) {
  // the preconditions rope_llama3 asserts (packages/kernels/root.zig:645-648), reported instead
  if (head_dim <= 0 || head_dim % 2 != 0 || !(theta > 0.f) || !(factor > 0.f) || !(low_freq_factor > 0.f) ||
      !(high_freq_factor > low_freq_factor) || original_max_position_embeddings <= 0 || T < 0 ||
      (T > 0 && (!positions || !cos_out || !sin_out)))
    return ncm_fail(NCM_EINVAL, "rope_tables_llama3: bad arguments");
  const RopeLlama3 l3{factor, low_freq_factor, high_freq_factor, original_max_position_embeddings};
  rope_tables_host(head_dim, theta, positions, static_cast<int>(T), cos_out, sin_out, &l3);
  return NCM_OK;
}

// ncm_attention_bf16 and its QK-norm variant: RoPE (or QK-norm then RoPE) and
// the V transpose, then the fused attention kernel
static int attention_entry(ncm_ctx_t* ctx, uint16_t* qkv, int64_t qkv_stride, const float* cos_t,
                           const float* sin_t, const uint16_t* q_norm, const uint16_t* k_norm, float eps,
                           uint16_t* out, int64_t T, int32_t heads, int32_t kv_heads, const ncm_mask_t* mask,
                           ncm_stream_t stream) {
  int rc = ctx_ok(ctx);
  if (rc) return rc;
  if (T <= 0 || T > INT32_MAX || T % 8 != 0 || heads <= 0 || kv_heads <= 0 || heads % kv_heads != 0 || !qkv || !out)
    return ncm_fail(NCM_EINVAL, "attention: bad shape (T=%lld must be a multiple of 8, heads %d, kv_heads %d)",
                    (long long)T, heads, kv_heads);
  if (qkv_stride < static_cast<int64_t>(heads + 2 * kv_heads) * 64 || qkv_stride % 8 != 0)
    return ncm_fail(NCM_EINVAL, "attention: qkv_stride %lld too small or not a multiple of 8", (long long)qkv_stride);
  if ((cos_t == nullptr) != (sin_t == nullptr)) return ncm_fail(NCM_EINVAL, "attention: give both cos and sin");
  if (!a16(qkv) || !a16(out)) return ncm_fail(NCM_EINVAL, "attention: buffers must be 16-byte aligned");
  if ((rc = check_mask(mask, T))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t vw = static_cast<int64_t>(kv_heads) * 64;
  WsCarver cv;
  const size_t o_vt = cv.take(2 * vw * T);
  uint8_t* ws = static_cast<uint8_t*>(ctx_workspace(ctx, cv.offset));
  if (ws == nullptr) return ncm_fail(NCM_ENOMEM, "attention: workspace allocation failed");
  uint16_t* vt = reinterpret_cast<uint16_t*>(ws + o_vt);
  {
    Launch _l(ctx, KID_DECODER_ELEMENTWISE, st);
    if (q_norm != nullptr)
      NCM_CUDA_TRY(launch_qk_norm_rope_bf16(qkv, qkv_stride, static_cast<int>(T), heads, kv_heads, q_norm, k_norm, eps,
                                            cos_t, sin_t, st));
    else if (cos_t != nullptr)
      NCM_CUDA_TRY(launch_rope_bf16(qkv, qkv_stride, static_cast<int>(T), heads + kv_heads, cos_t, sin_t, st));
    NCM_CUDA_TRY(launch_v_transpose(qkv, qkv_stride, static_cast<int64_t>(heads + kv_heads) * 64,
                                    static_cast<int>(T), static_cast<int>(vw), vt, st));
  }
  Launch _l(ctx, KID_ATTENTION, st);
  return attention_bf16(ctx, qkv, qkv_stride, vt, out, static_cast<int>(T), heads, kv_heads, mask->mode,
                        mask->prefix_length, mask->prefix_pad_mask, mask->level_lengths, mask->num_levels,
                        mask->sliding_window, st);
}

int ncm_attention_bf16(ncm_ctx_t* ctx, uint16_t* qkv, int64_t qkv_stride, const float* cos_t, const float* sin_t,
                       uint16_t* out, int64_t T, int32_t heads, int32_t kv_heads, const ncm_mask_t* mask,
                       ncm_stream_t stream) {
  return attention_entry(ctx, qkv, qkv_stride, cos_t, sin_t, nullptr, nullptr, 0.f, out, T, heads, kv_heads, mask,
                         stream);
}

int ncm_attention_qk_norm_bf16(ncm_ctx_t* ctx, uint16_t* qkv, int64_t qkv_stride, const float* cos_t,
                               const float* sin_t, const uint16_t* q_norm, const uint16_t* k_norm, float eps,
                               uint16_t* out, int64_t T, int32_t heads, int32_t kv_heads, const ncm_mask_t* mask,
                               ncm_stream_t stream) {
  if (int rc = ctx_ok(ctx)) return rc;
  if (q_norm == nullptr || k_norm == nullptr)
    return ncm_fail(NCM_EINVAL, "attention: give both q_norm and k_norm (attention_impl takes both or neither)");
  if (!a16(q_norm) || !a16(k_norm)) return ncm_fail(NCM_EINVAL, "attention: norm weights must be 16-byte aligned");
  if (!(eps >= 0.f)) return ncm_fail(NCM_EINVAL, "attention: eps must be a non-negative number");
  return attention_entry(ctx, qkv, qkv_stride, cos_t, sin_t, q_norm, k_norm, eps, out, T, heads, kv_heads, mask,
                         stream);
}

int ncm_qkv_projection_rope(ncm_ctx_t* ctx, const uint16_t* x, const uint16_t* w, const uint16_t* bias,
                            const float* cos_t, const float* sin_t, uint16_t* qkv, uint16_t* vt, int64_t T,
                            int64_t hidden, int32_t heads, int32_t kv_heads, ncm_stream_t stream) {
  int rc = ctx_ok(ctx);
  if (rc) return rc;
  if (T <= 64 || T > INT32_MAX || hidden <= 0 || hidden % 8 != 0 || heads <= 0 || kv_heads <= 0)
    return ncm_fail(NCM_EINVAL, "qkv_projection_rope: bad shape (T=%lld must exceed 64, hidden %lld)", (long long)T,
                    (long long)hidden);
  if (!x || !w || !cos_t || !sin_t || !qkv || !vt) return ncm_fail(NCM_EINVAL, "qkv_projection_rope: null buffer");
  if (!a16(x) || !a16(w) || !a16(qkv) || (bias && !a16(bias)))
    return ncm_fail(NCM_EINVAL, "qkv_projection_rope: buffers must be 16-byte aligned");
  if (!a16(cos_t) || !a16(sin_t)) return ncm_fail(NCM_EINVAL, "qkv_projection_rope: tables must be 16-byte aligned");
  const int64_t N = static_cast<int64_t>(heads + 2 * kv_heads) * 64;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  WsCarver cv;
  const size_t o_c = cv.take(2 * T * 64), o_s = cv.take(2 * T * 64);
  uint8_t* ws = static_cast<uint8_t*>(ctx_workspace(ctx, cv.offset));
  if (ws == nullptr) return ncm_fail(NCM_ENOMEM, "qkv_projection_rope: workspace allocation failed");
  uint16_t* cb = reinterpret_cast<uint16_t*>(ws + o_c);
  uint16_t* sb = reinterpret_cast<uint16_t*>(ws + o_s);
  {
    Launch _l(ctx, KID_CAST, st);
    NCM_CUDA_TRY(launch_f32_to_bf16(cos_t, cb, T * 64, st));
    NCM_CUDA_TRY(launch_f32_to_bf16(sin_t, sb, T * 64, st));
  }
  return linear_qkv_rope(ctx, x, w, bias, qkv, vt, cb, sb, T, hidden, N, static_cast<int64_t>(heads + kv_heads) * 64,
                         st);
}

int ncm_ncm_forward(ncm_ctx_t* ctx, const ncm_decoder_config_t* cfg, const ncm_decoder_weights_t* W,
                    const uint16_t* inputs, uint16_t* out, ncm_stream_t stream) {
  int rc = ctx_ok(ctx);
  if (rc) return rc;
  if (!cfg || !W || !inputs || !out) return ncm_fail(NCM_EINVAL, "ncm_forward: null argument");
  const ncm_mask_t& m = cfg->mask;
  // causal mode is ncm_model's source_causal: the levels still give the RoPE
  // positions and the level embeddings
  if (m.num_levels <= 0 || m.num_levels > 32 || m.prefix_length < 0)
    return ncm_fail(NCM_EINVAL, "ncm_forward: num_levels %d or prefix_length %d out of range", m.num_levels,
                    m.prefix_length);
  int64_t T = m.prefix_length;
  for (int i = 0; i < m.num_levels; ++i) {
    if (m.level_lengths[i] <= 0) return ncm_fail(NCM_EINVAL, "ncm_forward: level %d is empty", i);
    T += m.level_lengths[i];
  }
  const int64_t Hd = cfg->hidden_size, V = cfg->vq_width, F = cfg->intermediate_size;
  const int H = static_cast<int>(cfg->num_attention_heads), Hkv = static_cast<int>(cfg->num_key_value_heads);
  if (cfg->head_dim != 64) return ncm_fail(NCM_EINVAL, "ncm_forward: head_dim must be 64");
  if (cfg->rope_type != 0 &&
      (cfg->rope_type != 1 || !(cfg->rope_factor > 0.f) || !(cfg->rope_low_freq_factor > 0.f) ||
       !(cfg->rope_high_freq_factor > cfg->rope_low_freq_factor) || cfg->rope_original_max_position_embeddings <= 0))
    return ncm_fail(NCM_EINVAL, "ncm_forward: rope_type %d or its llama3 parameters are invalid", cfg->rope_type);
  if (Hd <= 0 || V <= 0 || F <= 0 || Hd % 8 || V % 8 || F % 8 || H <= 0 || Hkv <= 0 || H % Hkv)
    return ncm_fail(NCM_EINVAL, "ncm_forward: bad dimensions");
  if ((rc = check_mask(&m, T))) return rc;
  if (T % 8 != 0) return ncm_fail(NCM_EINVAL, "ncm_forward: sequence length %lld must be a multiple of 8", (long long)T);
  if (W->num_layers <= 0 || W->layers == nullptr || !W->input_projection || !W->input_projection_bias ||
      !W->final_norm || (cfg->use_level_encoding && !W->level_embedding))
    return ncm_fail(NCM_EINVAL, "ncm_forward: missing weights");
  for (int l = 0; l < W->num_layers; ++l) {
    const auto& L = W->layers[l];
    if (!L.ln_1 || !L.qkv || !L.o || !L.ln_2 || !L.gate_up || !L.down)
      return ncm_fail(NCM_EINVAL, "ncm_forward: layer %d is missing a weight", l);
    if ((L.q_norm == nullptr) != (L.k_norm == nullptr))
      return ncm_fail(NCM_EINVAL, "ncm_forward: layer %d needs both q_norm and k_norm or neither", l);
    if ((L.q_norm && !a16(L.q_norm)) || (L.k_norm && !a16(L.k_norm)))
      return ncm_fail(NCM_EINVAL, "ncm_forward: layer %d norm weights must be 16-byte aligned", l);
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t QKV = static_cast<int64_t>(H + 2 * Hkv) * 64;
  WsCarver cv;
  const size_t o_h = cv.take(2 * T * Hd), o_n = cv.take(2 * T * Hd), o_qkv = cv.take(2 * T * QKV);
  const size_t o_vt = cv.take(2 * T * Hkv * 64), o_ctx = cv.take(2 * T * H * 64), o_a = cv.take(2 * T * Hd);
  const bool fused_swiglu = T > 64 && F % 128 == 0;
  const size_t o_gu = fused_swiglu ? 0 : cv.take(2 * T * 2 * F), o_act = cv.take(2 * T * F);
  // post-upsample convolutions: convolved input rows, one level's padded copy, one packed kernel
  const bool post_conv = W->post_conv_weight != nullptr;
  if (post_conv != (W->post_conv_bias != nullptr))
    return ncm_fail(NCM_EINVAL, "ncm_forward: pass both post-conv weight and bias, or neither");
  if (post_conv && !a16(W->post_conv_bias))
    return ncm_fail(NCM_EINVAL, "ncm_forward: post-conv bias must be 16-byte aligned");
  const int64_t Vp = (V + 63) / 64 * 64;
  int64_t max_level = 0;
  for (int i = 0; i < m.num_levels; ++i) max_level = std::max<int64_t>(max_level, m.level_lengths[i]);
  const size_t o_xin = post_conv ? cv.take(2 * T * V) : 0;
  const size_t o_cpad = post_conv ? cv.take(2 * (max_level + 2) * Vp) : 0;
  const size_t o_cw = post_conv ? cv.take(2 * V * 3 * Vp) : 0;
  uint8_t* ws = static_cast<uint8_t*>(ctx_workspace(ctx, cv.offset));
  if (ws == nullptr) return ncm_fail(NCM_ENOMEM, "ncm_forward: workspace allocation failed");
  uint16_t* h = reinterpret_cast<uint16_t*>(ws + o_h);
  uint16_t* nrm = reinterpret_cast<uint16_t*>(ws + o_n);
  uint16_t* qkv = reinterpret_cast<uint16_t*>(ws + o_qkv);
  uint16_t* vt = reinterpret_cast<uint16_t*>(ws + o_vt);
  uint16_t* ctxb = reinterpret_cast<uint16_t*>(ws + o_ctx);
  uint16_t* gu = reinterpret_cast<uint16_t*>(ws + o_gu);
  uint16_t* act = reinterpret_cast<uint16_t*>(ws + o_act);
  (void)o_a;

  // RoPE tables at per-level restarting positions (ncm_position.fill_level_positions)
  // and each row's level: built on the host once per configuration and kept
  // on the device, so repeated forwards do no host work or synchronisation.
  uint64_t key = 1469598103934665603ull;
  auto mix = [&key](uint64_t v) { key = (key ^ v) * 1099511628211ull; };
  mix(static_cast<uint64_t>(T));
  uint32_t theta_bits;
  std::memcpy(&theta_bits, &cfg->rope_theta, 4);
  mix(theta_bits);
  mix(static_cast<uint64_t>(m.prefix_length));
  mix(static_cast<uint64_t>(cfg->use_level_encoding));
  mix(static_cast<uint64_t>(cfg->rope_type));
  if (cfg->rope_type == 1) {
    uint32_t b[3];
    std::memcpy(&b[0], &cfg->rope_factor, 4);
    std::memcpy(&b[1], &cfg->rope_low_freq_factor, 4);
    std::memcpy(&b[2], &cfg->rope_high_freq_factor, 4);
    for (uint32_t v : b) mix(v);
    mix(static_cast<uint64_t>(cfg->rope_original_max_position_embeddings));
  }
  for (int i = 0; i < m.num_levels; ++i) mix(static_cast<uint64_t>(m.level_lengths[i]));
  if (key != ctx->rope_key || ctx->rope_cos == nullptr) {
    std::vector<int> pos(T), lev(T);
    int64_t t = 0;
    for (; t < m.prefix_length; ++t) pos[t] = static_cast<int>(t), lev[t] = -1;
    for (int i = 0; i < m.num_levels; ++i)
      for (int p = 0; p < m.level_lengths[i]; ++p, ++t) pos[t] = p, lev[t] = cfg->use_level_encoding ? i : -1;
    std::vector<float> ch(T * 64), sh(T * 64);
    const RopeLlama3 l3{cfg->rope_factor, cfg->rope_low_freq_factor, cfg->rope_high_freq_factor,
                        cfg->rope_original_max_position_embeddings};
    rope_tables_host(64, cfg->rope_theta, pos.data(), static_cast<int>(T), ch.data(), sh.data(),
                     cfg->rope_type == 1 ? &l3 : nullptr);
    NCM_CUDA_TRY(cudaStreamSynchronize(st));  // no forward in flight still reads the old tables
    if (T > ctx->rope_rows) {
      cudaFree(ctx->rope_cos);
      cudaFree(ctx->rope_sin);
      cudaFree(ctx->rope_cos_bf);
      cudaFree(ctx->rope_sin_bf);
      cudaFree(ctx->rope_row_level);
      ctx->rope_cos = ctx->rope_sin = nullptr;
      ctx->rope_cos_bf = ctx->rope_sin_bf = nullptr;
      ctx->rope_row_level = nullptr;
      ctx->rope_rows = 0;
      NCM_CUDA_TRY(cudaMalloc(&ctx->rope_cos, 4 * T * 64));
      NCM_CUDA_TRY(cudaMalloc(&ctx->rope_sin, 4 * T * 64));
      NCM_CUDA_TRY(cudaMalloc(&ctx->rope_cos_bf, 2 * T * 64));
      NCM_CUDA_TRY(cudaMalloc(&ctx->rope_sin_bf, 2 * T * 64));
      NCM_CUDA_TRY(cudaMalloc(&ctx->rope_row_level, 4 * T));
      ctx->rope_rows = T;
    }
    NCM_CUDA_TRY(cudaMemcpy(ctx->rope_cos, ch.data(), 4 * T * 64, cudaMemcpyHostToDevice));
    NCM_CUDA_TRY(cudaMemcpy(ctx->rope_sin, sh.data(), 4 * T * 64, cudaMemcpyHostToDevice));
    {
      // bf16-rounded copies for the fused QKV epilogue (rotate_head rounds each table value)
      std::vector<uint16_t> cb(T * 64), sb(T * 64);
      for (int64_t i = 0; i < T * 64; ++i) cb[i] = f32_to_bf16(ch[i]), sb[i] = f32_to_bf16(sh[i]);
      NCM_CUDA_TRY(cudaMemcpy(ctx->rope_cos_bf, cb.data(), 2 * T * 64, cudaMemcpyHostToDevice));
      NCM_CUDA_TRY(cudaMemcpy(ctx->rope_sin_bf, sb.data(), 2 * T * 64, cudaMemcpyHostToDevice));
    }
    NCM_CUDA_TRY(cudaMemcpy(ctx->rope_row_level, lev.data(), 4 * T, cudaMemcpyHostToDevice));
    ctx->rope_key = key;
  }
  const float* cosd = ctx->rope_cos;
  const float* sind = ctx->rope_sin;
  const int* row_level = ctx->rope_row_level;

  const int Ti = static_cast<int>(T);
  const float eps = cfg->rms_norm_epsilon;
  if (post_conv) {
    // ncm_model.zig:141-153: each level's rows get x + bias + conv(x) with that level's kernel
    uint16_t* xin = reinterpret_cast<uint16_t*>(ws + o_xin);
    uint16_t* cpad = reinterpret_cast<uint16_t*>(ws + o_cpad);
    uint16_t* cw = reinterpret_cast<uint16_t*>(ws + o_cw);
    NCM_CUDA_TRY(cudaMemcpyAsync(xin, inputs, 2 * T * V, cudaMemcpyDeviceToDevice, st));
    int64_t row0 = m.prefix_length;
    for (int i = 0; i < m.num_levels; ++i) {
      const int64_t n = m.level_lengths[i];
      SegMap map{};
      map.seg_len = static_cast<int>(n);
      map.nseg = 1;
      {
        Launch _l(ctx, KID_CAST, st);
        NCM_CUDA_TRY(launch_conv_repack(W->post_conv_weight + static_cast<size_t>(i) * V * V * 3, nullptr, cw, V, Vp,
                                        st));
        NCM_CUDA_TRY(launch_conv_pad(nullptr, inputs + row0 * V, cpad, map, V, Vp, st));
      }
      ConvEpilogue ep{};
      ep.x_bf16 = inputs + row0 * V;
      ep.out_bf16 = xin + row0 * V;
      ep.bias = W->post_conv_bias + i * V;
      ep.alpha = 1.f;
      ep.beta = 1.f;
      if ((rc = conv3_gemm(ctx, cpad, cw, map, Vp, V, ep, st))) return rc;
      row0 += n;
    }
    inputs = xin;
  }
  rc = linear_bf16(ctx, inputs, W->input_projection, W->input_projection_bias, h, nullptr, T, V, Hd, st);
  if (rc) return rc;
  if (cfg->use_level_encoding) {
    Launch _l(ctx, KID_DECODER_ELEMENTWISE, st);
    NCM_CUDA_TRY(launch_add_level_embedding(h, W->level_embedding, row_level, Ti, static_cast<int>(Hd), st));
  }
  for (int l = 0; l < W->num_layers; ++l) {
    const auto& L = W->layers[l];
    {
      Launch _l(ctx, KID_DECODER_ELEMENTWISE, st);
      NCM_CUDA_TRY(launch_rms_norm_bf16(h, L.ln_1, nullptr, nrm, Ti, static_cast<int>(Hd), eps, st));
    }
    if (L.q_norm != nullptr) {
      // QK-norm sits between the projection and RoPE (ncm_model.zig:271-272,
      // root.zig:500-530), so the RoPE epilogue does not apply
      if ((rc = linear_bf16(ctx, nrm, L.qkv, L.qkv_bias, qkv, nullptr, T, Hd, QKV, st))) return rc;
      Launch _l(ctx, KID_DECODER_ELEMENTWISE, st);
      NCM_CUDA_TRY(launch_qk_norm_rope_bf16(qkv, QKV, Ti, H, Hkv, L.q_norm, L.k_norm, eps, cosd, sind, st));
      NCM_CUDA_TRY(launch_v_transpose(qkv, QKV, static_cast<int64_t>(H + Hkv) * 64, Ti, Hkv * 64, vt, st));
    } else if (T > 64) {
      // RoPE and the V transpose in the projection's epilogue
      if ((rc = linear_qkv_rope(ctx, nrm, L.qkv, L.qkv_bias, qkv, vt, ctx->rope_cos_bf, ctx->rope_sin_bf, T, Hd, QKV,
                                static_cast<int64_t>(H + Hkv) * 64, st)))
        return rc;
    } else {
      if ((rc = linear_bf16(ctx, nrm, L.qkv, L.qkv_bias, qkv, nullptr, T, Hd, QKV, st))) return rc;
      Launch _l(ctx, KID_DECODER_ELEMENTWISE, st);
      NCM_CUDA_TRY(launch_rope_bf16(qkv, QKV, Ti, H + Hkv, cosd, sind, st));
      NCM_CUDA_TRY(launch_v_transpose(qkv, QKV, static_cast<int64_t>(H + Hkv) * 64, Ti, Hkv * 64, vt, st));
    }
    {
      Launch _l(ctx, KID_ATTENTION, st);
      if ((rc = attention_bf16(ctx, qkv, QKV, vt, ctxb, Ti, H, Hkv, m.mode, m.prefix_length, m.prefix_pad_mask,
                               m.level_lengths, m.num_levels, m.sliding_window, st)))
        return rc;
    }
    // h = bf16(h + bf16(ctx . O^T + b)) in the projection's epilogue
    if ((rc = linear_bf16_ex(ctx, ctxb, L.o, L.o_bias, h, nullptr, T, static_cast<int64_t>(H) * 64, Hd, st, 2, 0)))
      return rc;
    {
      Launch _l(ctx, KID_DECODER_ELEMENTWISE, st);
      NCM_CUDA_TRY(launch_rms_norm_bf16(h, L.ln_2, nullptr, nrm, Ti, static_cast<int>(Hd), eps, st));
    }
    if (fused_swiglu) {
      // act = bf16(bf16(silu(g)) * u) straight from the gate|up projection's epilogue
      if ((rc = linear_bf16_ex(ctx, nrm, L.gate_up, nullptr, act, nullptr, T, Hd, 2 * F, st, 1, F))) return rc;
    } else {
      if ((rc = linear_bf16(ctx, nrm, L.gate_up, nullptr, gu, nullptr, T, Hd, 2 * F, st))) return rc;
      Launch _l(ctx, KID_DECODER_ELEMENTWISE, st);
      NCM_CUDA_TRY(launch_silu_mul_bf16(gu, act, Ti, static_cast<int>(F), st));
    }
    // h = bf16(h + bf16(act . down^T)) in the projection's epilogue
    if ((rc = linear_bf16_ex(ctx, act, L.down, nullptr, h, nullptr, T, F, Hd, st, 2, 0))) return rc;
  }
  Launch _l(ctx, KID_DECODER_ELEMENTWISE, st);
  NCM_CUDA_TRY(launch_rms_norm_bf16(h, W->final_norm, W->final_norm_bias, out, Ti, static_cast<int>(Hd), eps, st));
  return NCM_OK;
}

}  // extern "C"
