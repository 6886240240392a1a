/*
 * ncm_oracle.h — CPU oracle for the ncmorph_b200 parity tests and the timed
 * CPU baseline. TEST INFRASTRUCTURE ONLY: the product library never links,
 * loads or calls this code; only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg do, as the checker.
 *
 * Each function restates the arithmetic of one ncmorph function (cited by
 * file:line relative to the ncmorph repository root) in plain C++, in the
 * same operation order, so that results are bit-identical to the reference
 * where the reference defines them:
 *   - bf16 conversion        packages/bf16/root.zig:17-37
 *   - linears                packages/kernels/root.zig:25-148
 *   - norms / activations    packages/kernels/root.zig:150-301
 *   - RoPE, masks, attention packages/kernels/root.zig:303-674
 *   - NCM masks / positions  src/ncm_mask.zig:10-46, src/ncm_position.zig:11-118
 *   - post-upsample conv     src/ncm_model.zig:296-326
 * The RVQ functions (orc_rvq_*, orc_pool_avg, orc_tokenizer_*) restate the
 * written specification research/reference/vq_forward_semantics.md:59-82,
 * because ncmorph has no RVQ code (ROADMAP.md:257-259): their parity is
 * anchored on torch's F.interpolate(mode="area") and argmin semantics, not
 * on reference test vectors.
 */
#ifndef NCM_ORACLE_H
#define NCM_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- bf16 (packages/bf16/root.zig:17-37) */
uint16_t orc_bf16_from_f32(float v);
float orc_bf16_to_f32(uint16_t b);
void orc_bf16_from_f32_n(const float* x, uint16_t* y, size_t n);
void orc_round_bf16_n(const float* x, float* y, size_t n);

/* ---- linears */
void orc_matmul(const float* in, const float* w, float* out, size_t T, size_t in_w, size_t out_w);
void orc_matmul_reference(const float* in, const float* w, float* out, size_t T, size_t in_w, size_t out_w);
/* bias may be NULL (matmul_bf16) */
void orc_matmul_bf16(const float* in, const float* w, const float* bias, float* out, size_t T, size_t in_w,
                     size_t out_w);
/* same arithmetic, rows split over `threads` OpenMP threads (timed baseline) */
void orc_matmul_bf16_mt(const float* in, const float* w, const float* bias, float* out, size_t T, size_t in_w,
                        size_t out_w, int threads);

/* ---- norms and activations */
float orc_sum_squares_pinned(const float* x, size_t n);
void orc_rms_norm(const float* in, const float* w, float* out, size_t n, float eps);
void orc_rms_norm_bf16(const float* in, const float* w, float* out, size_t n, float eps);
void orc_silu(const float* in, float* out, size_t n);
void orc_silu_bf16(const float* in, float* out, size_t n);
void orc_softmax(const float* in, float* out, size_t n);
void orc_rms_norm_rows(const float* in, const float* w, const float* bias, float* out, size_t rows, size_t width,
                       float eps);

/* ---- RoPE and masks */
void orc_rope_default(size_t head_dim, float theta, size_t positions, float* inv_freq, float* cos_t, float* sin_t);
void orc_rope_tables(const float* inv_freq, size_t half_dim, size_t positions, float* cos_t, float* sin_t);
void orc_rope_llama3(size_t head_dim, float theta, float factor, float low_ff, float high_ff, size_t orig_max,
                     float* inv_freq);
/* window <= 0 means no sliding window; output [Q*K] as bytes (1 = allowed) */
void orc_causal_mask(const size_t* qpos, size_t nq, const size_t* kpos, size_t nk, long window, uint8_t* out);
int orc_block_diagonal_mask(size_t prefix, const size_t* levels, size_t nlevels, const uint8_t* pad_mask,
                            size_t pad_len, uint8_t* out, size_t out_len);
/* block-causal variant: a level also sees every earlier (coarser) level */
int orc_block_causal_mask(size_t prefix, const size_t* levels, size_t nlevels, const uint8_t* pad_mask,
                          size_t pad_len, uint8_t* out, size_t out_len);
int orc_fill_level_positions(size_t prefix, const size_t* levels, size_t nlevels, size_t* out, size_t out_len);
int orc_apply_post_upsample_conv(float* x, const float* w, const float* b, size_t rows, size_t width);

/* ---- attention (packages/kernels/root.zig:450-581); null-able weights as in attention_weights_t */
typedef struct orc_attention_weights {
  const float* q_w;
  const float* q_b;
  const float* k_w;
  const float* k_b;
  const float* v_w;
  const float* v_b;
  const float* q_norm;
  const float* k_norm;
  const float* o_w;
  const float* o_b;
} orc_attention_weights_t;

int orc_attention(const float* in, const orc_attention_weights_t* w, size_t T, size_t hidden, size_t heads,
                  size_t kv_heads, size_t head_dim, float eps, const float* cos_t, const float* sin_t,
                  const uint8_t* mask, float* out, int bf16_mode, float* context_trace);

/* attention_impl's core for a subset of query rows (Q projected and rotated
 * [nrows, H*hd]; K rotated and V [T, Hkv*hd]; mask rows [nrows, T]); context
 * rows [nrows, H*hd], the same bits as orc_attention's rows. */
int orc_attention_core_rows(const float* Q, const float* Kt, const float* V, const uint8_t* mask, size_t nrows,
                            size_t T, size_t H, size_t Hkv, size_t hd, float* ctx, int bf16_mode, int threads);
/* rotate_head over every head of n rows, each row with its own table row. */
void orc_rotate_rows(float* x, size_t n, size_t heads, size_t hd, const float* cos_t, const float* sin_t,
                     int bf16_mode);

/* ---- RVQ (spec restatement) */
void orc_code_sqnorm(const uint16_t* cb, float* out, size_t K, size_t D);
/* One level. If codes_in is non-NULL the residual is advanced with those codes
 * (teacher forcing) while best_out still receives the oracle's own argmin.
 * rel_gap (nullable): (d2 - d1) / ||bf16(r) - e_best||^2 per row. */
void orc_rvq_level(float* resid, const uint16_t* cb, const float* sqnorm, const int32_t* codes_in,
                   int32_t* best_out, float* rel_gap, size_t N, size_t D, size_t K, int threads);
void orc_rvq_decode(const int32_t* codes, const uint16_t* cbs, size_t L, float* recon_f32, size_t N, size_t D,
                    size_t K);
void orc_pool_avg(const float* x, float* y, size_t B, size_t T, size_t D, size_t f);
void orc_group_norm(const float* x, float* y, size_t B, size_t T, size_t C, size_t G, float eps);
void orc_conv_down4(const float* x, const float* w, const float* b, float* y, size_t B, size_t L, size_t C);
void orc_conv_up4(const float* x, const float* w, const float* b, float* y, size_t B, size_t L, size_t C);
void orc_ema(const float* u, const int32_t* codes, size_t N, size_t D, size_t K, float* ema_count, float* ema_sum,
             float* codebook, float decay, float eps, float* counts_out, float* sums_out);
void orc_tied_head(const float* z, const uint16_t* cb, const float* esq_in, const float* bias, float log_inv_T,
                   float* logits, int32_t* codes, float* gap, size_t T, size_t d, size_t K);
void orc_upsample(const float* q, float* out, size_t B, size_t Tq, size_t T, size_t D, int mode);
void orc_conv1d_k3(const float* x_op, const float* x_blend, const float* w, const float* b, float* out, size_t rows,
                   size_t width, const size_t* seg_lengths, size_t nseg, float alpha, float beta);
void orc_scale_update_ex(const int32_t* codes, const uint16_t* cbs, size_t L, float* resid, float* acc, size_t B,
                         size_t T, size_t D, size_t K, size_t f, int mode, const float* phi_w, const float* phi_b,
                         float ratio);
void orc_scale_update(const int32_t* codes, const uint16_t* cbs, size_t L, float* resid, float* recon, size_t B,
                      size_t T, size_t D, size_t K, size_t f);

#ifdef __cplusplus
}
#endif

#endif
