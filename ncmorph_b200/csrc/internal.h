// Host-side internals shared by the library's translation units: the context
// object, its device workspace, tensor-map encoding and kernel launchers.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <utility>
#include <vector>

#include "common.cuh"

namespace ncm {
// Kernel families counted (always) and timed (when profiling is enabled).
enum KernelId {
  KID_RVQ_ARGMIN = 0,
  KID_RVQ_APPLY,
  KID_LINEAR,
  KID_DECODE,
  KID_SQNORM,
  KID_POOL,
  KID_SCALE_UPDATE,
  KID_CAST,
  KID_ATTENTION,
  KID_DECODER_ELEMENTWISE,
  KID_CONV,
  KID_UPSAMPLE,
  KID_COUNT
};
extern const char* const kKernelNames[KID_COUNT];

struct ProfState {
  bool on = false;
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> events[KID_COUNT];
  size_t used[KID_COUNT] = {};
  long long launches[KID_COUNT] = {};
};
}  // namespace ncm

struct ncm_ctx {
  int device = 0;
  int num_sms = 0;
  int* d_err = nullptr;      // device error word (bit flags, see ptx.cuh)
  void* ws = nullptr;        // growable device workspace
  size_t ws_bytes = 0;
  // host staging for the *_host_f32 entry points
  void* h_stage = nullptr;
  size_t h_stage_bytes = 0;
  ncm::ProfState prof;
  // copy streams and events of the host-buffer pipeline (created on first use)
  cudaStream_t copy_in = nullptr;
  cudaStream_t copy_out = nullptr;
  cudaEvent_t ev_in[2] = {nullptr, nullptr};
  cudaEvent_t ev_done[2] = {nullptr, nullptr};
  cudaEvent_t ev_out[2] = {nullptr, nullptr};
  // RoPE tables and per-row levels of the last NCM forward configuration
  uint64_t rope_key = 0;
  float* rope_cos = nullptr;
  float* rope_sin = nullptr;
  uint16_t* rope_cos_bf = nullptr;  // the same tables rounded to bf16 (fused QKV epilogue)
  uint16_t* rope_sin_bf = nullptr;
  int* rope_row_level = nullptr;
  int64_t rope_rows = 0;
  // split-fixup arrival counters of the RVQ argmin kernel (kept zero between launches)
  int* rvq_counters = nullptr;
  int64_t rvq_counter_len = 0;
  // f32 partial sums of the split-K skinny GEMM (its own buffer: the callers'
  // activations may live in the workspace, which must not move under them)
  float* kpart = nullptr;
  size_t kpart_bytes = 0;
  // pinned staging buffers and their events of the checkpoint loader (first use)
  void* load_h[2] = {nullptr, nullptr};
  cudaEvent_t load_ev[2] = {nullptr, nullptr};
  size_t load_bytes = 0;
  // NCCL communicator bound by ncm_ctx_comm_init (row-sharded entry points)
  void* comm = nullptr;
  int comm_rank = 0;
  int comm_size = 1;
};

namespace ncm {

// Counts one launch of kernel family `id` on `stream` and, while profiling is
// enabled, brackets it with CUDA events recorded on that stream.
class Launch {
 public:
  Launch(ncm_ctx* ctx, KernelId id, cudaStream_t stream);
  ~Launch();
  Launch(const Launch&) = delete;
  Launch& operator=(const Launch&) = delete;

 private:
  ncm_ctx* ctx_;
  KernelId id_;
  cudaStream_t stream_;
  cudaEvent_t stop_ = nullptr;
};

// Launch with the programmatic stream-serialization attribute (and a cluster
// dimension when cluster_x > 1): the kernel may begin while its predecessor on
// the stream drains; it calls pdl_wait() before touching that predecessor's data.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       int cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  int n = 1;
  if (cluster_x > 1) {
    at[1].id = cudaLaunchAttributeClusterDimension;
    at[1].val.clusterDim.x = cluster_x;
    at[1].val.clusterDim.y = 1;
    at[1].val.clusterDim.z = 1;
    n = 2;
  }
  cfg.attrs = at;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Carves consecutive 256-byte-aligned regions out of the context workspace.
struct WsCarver {
  size_t offset = 0;
  size_t take(size_t bytes) {
    const size_t at = offset;
    offset += (bytes + 255) & ~static_cast<size_t>(255);
    return at;
  }
};

// Process-wide per-device state that host threads driving different GPUs
// share (one bit per device index below 64): a kernel's shared-memory opt-in
// is per device, so it is set once per device, from any thread.
class DeviceFlags {
 public:
  bool test(int dev) const { return dev >= 0 && dev < 64 && (bits_.load(std::memory_order_acquire) >> dev) & 1ull; }
  void set(int dev) {
    if (dev >= 0 && dev < 64) bits_.fetch_or(1ull << dev, std::memory_order_release);
  }

 private:
  std::atomic<unsigned long long> bits_{0};
};

// Ensures the workspace holds at least `bytes`; returns its base or nullptr.
void* ctx_workspace(ncm_ctx* ctx, size_t bytes);

// Builds a 2-D bf16 tensor map over a row-major [rows, cols] matrix with a
// box of [box_rows, 64] and 128-byte swizzling. Returns false on failure.
bool make_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows);

// Same, over rows `row_stride` elements apart (a column slice of a wider matrix).
bool make_tmap_bf16_2d_strided(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                               uint64_t row_stride, uint32_t box_rows);

// ---- decoder pieces (decoder.cu, attention.cu)
cudaError_t launch_rms_norm_bf16(const uint16_t* x, const uint16_t* w, const uint16_t* b, uint16_t* y, int rows,
                                 int width, float eps, cudaStream_t st);
cudaError_t launch_rope_bf16(uint16_t* qkv, long long stride, int T, int heads_qk, const float* c, const float* s,
                             cudaStream_t st);
// per-head RMSNorm (q_norm on the Q heads, k_norm on the K heads; either
// null skips it) then RoPE (skipped when c is null), in place, bf16 mode
cudaError_t launch_qk_norm_rope_bf16(uint16_t* qkv, long long stride, int T, int heads, int kv_heads,
                                     const uint16_t* q_norm, const uint16_t* k_norm, float eps, const float* c,
                                     const float* s, cudaStream_t st);
cudaError_t launch_v_transpose(const uint16_t* qkv, long long stride, long long voff, int T, int vwidth, uint16_t* vt,
                               cudaStream_t st);
cudaError_t launch_silu_mul_bf16(const uint16_t* gu, uint16_t* out, int T, int F, cudaStream_t st);
cudaError_t launch_add_bf16(uint16_t* h, const uint16_t* a, long long n, cudaStream_t st);
cudaError_t launch_add_level_embedding(uint16_t* h, const uint16_t* emb, const int* row_level, int T, int width,
                                       cudaStream_t st);
cudaError_t launch_embedding_gather(const uint16_t* table, int vocab, int width, const int32_t* ids, int T,
                                    uint16_t* out, int* err, cudaStream_t st);
// Llama 3 frequency scaling (rope_llama3's parameters).
struct RopeLlama3 {
  float factor, low_freq_factor, high_freq_factor;
  int64_t original_max_position_embeddings;
};
void rope_inv_freq(int head_dim, float theta, const RopeLlama3* llama3, float* inv);
void rope_tables_host(int head_dim, float theta, const int* positions, int T, float* cos_out, float* sin_out,
                      const RopeLlama3* llama3 = nullptr);
// Fused masked attention over the Q and K columns of fused QKV rows (row
// stride qkv_stride elements) and V transposed to [Hkv*64, T]; head_dim 64.
// mode 0 causal (window > 0: keys q - window < k <= q), 1 block-diagonal,
// 2 block-causal.
int attention_bf16(ncm_ctx* ctx, const uint16_t* qkv, int64_t qkv_stride, const uint16_t* vt, uint16_t* out, int T,
                   int H, int Hkv, int mode, int prefix, unsigned long long pad_mask, const int* level_lens,
                   int nlev, int window, cudaStream_t stream);

// ---- RVQ launchers (rvq.cu)
struct RvqPartial {
  float d;
  int idx;
};

// Plans how many code splits one level uses; returns workspace bytes needed
// for the partial results (0 when no split).
// pair = 1: CTA pairs share each MMA (units of 256 rows, splits = 1); the
// codebook tensor map then needs a 128-row box (rvq_codebook_box_rows).
struct RvqPlan {
  int row_blocks, code_tiles, splits, tiles_per_split, n_units, grid;
  size_t partial_bytes;
  int pair;
};
RvqPlan rvq_plan(int num_sms, int64_t N, int64_t K, bool allow_pair = false);
inline uint32_t rvq_codebook_box_rows(const RvqPlan& p) { return p.pair ? 128u : 256u; }

// Residual update done inside the distance kernel (only when the plan has
// one code split): resid = (src_bf16 ? f32(src_bf16) : resid) - e[code],
// shadow = bf16(resid) when shadow is non-null.
struct RvqFusedUpdate {
  float* resid;
  const uint16_t* src_bf16;
  uint16_t* shadow;
  const uint16_t* codebook;
};

// Optional top-2 gap output: gap[n] = (d2 - d1) / (a2[n] + d1) with d1 <= d2
// the two smallest GEMM distances of row n and a2 = ||bf16(r_n)||^2;
// part_d2 ([splits, N] f32) carries each split's second-smallest distance.
struct RvqTop2 {
  float* gap;
  const float* a2;
  float* part_d2;
};

// argmin_k (sqnorm[k] - 2 a_n . e_k) over bf16 rows `a` [N,D] (via tmA) and
// (with mul_dev: argmin_k fmaf(*mul_dev, a_n . e_k, sqnorm[k]), the tied head's form)
// With counters (and no top2) a split plan merges its splits inside the
// kernel (the last CTA to finish a row block), writes the final codes and
// applies `fu`; rvq_apply_kernel is then not needed.
// codebook `e` [K,D] (via tmB). Writes codes (splits == 1) or partials, and
// applies `fu` when given and the plan has one split.
cudaError_t launch_rvq_argmin(const RvqPlan& plan, const CUtensorMap& tmA, const CUtensorMap& tmB,
                              const float* sqnorm, int32_t* codes, RvqPartial* part, int* err, int64_t N,
                              int64_t D, int64_t K, cudaStream_t stream, const RvqFusedUpdate* fu = nullptr,
                              const RvqTop2* top2 = nullptr, const float* mul_dev = nullptr,
                              int* counters = nullptr);
// Per row block arrival counters of the split fixup (zeroed, kept in the
// context, grown on demand); nullptr if the allocation fails.
int* rvq_counters(ncm_ctx* ctx, int64_t row_blocks);

// Final code per row (reducing partials when splits > 1), then
// resid = (src_bf16 ? f32(src_bf16) : resid) - e[code]; shadow = bf16(resid).
cudaError_t launch_rvq_apply(const RvqPlan& plan, const RvqPartial* part, int32_t* codes, const uint16_t* src_bf16,
                             float* resid, uint16_t* shadow, const uint16_t* codebook, int* err, int64_t N,
                             int64_t D, int64_t K, bool update, cudaStream_t stream, const RvqTop2* top2 = nullptr);

cudaError_t launch_code_sqnorm(const uint16_t* codebook, float* sqnorm, int64_t K, int64_t D, cudaStream_t stream);

// Every level of a small encode in one launch (rvq_levels.cu): one cluster of
// `cluster` CTAs per 128-row block, CTA r holding code tiles [r * tpc, ...)
// and residual columns [r * slice, ...). Applies when the row blocks cannot
// fill half the SMs (one level per launch would split the code range).
struct RvqLevelsPlan {
  int row_blocks, cluster, tpc, code_tiles, slice;
  int reg;  // the residual slice stays in registers and the kernel writes the reconstruction
};
bool rvq_levels_plan(int num_sms, int64_t N, int64_t D, int64_t K, int L, RvqLevelsPlan* out);
// codes [L, N], resid (f32; holds the final residual with keep_resid),
// shadow (bf16 scratch [N, D]); x [N, D] bf16 rows. With plan.reg the
// kernel also writes recon (bf16 [N, D], nullable); otherwise the caller
// decodes.
cudaError_t launch_rvq_levels(const RvqLevelsPlan& plan, const uint16_t* x, const uint16_t* codebooks,
                              const float* sqnorms, int L, int32_t* codes, float* resid, bool keep_resid,
                              uint16_t* shadow, uint16_t* recon, int* err, int64_t N, int64_t D, int64_t K,
                              cudaStream_t stream);
cudaError_t launch_rvq_decode(const int32_t* codes, const uint16_t* codebooks, int L, uint16_t* recon_bf16,
                              float* recon_f32, int64_t N, int64_t D, int64_t K, int* err, cudaStream_t stream);
cudaError_t launch_pool_avg(const float* x, float* y, uint16_t* y_bf16, int64_t B, int64_t T, int64_t D, int f,
                            cudaStream_t stream);
// Scale s of the multiscale driver: q_out[p] = sum_l e_l[codes[l,p]]; with
// update_r also resid -= up(q) over the f rows of each pooled row, and when
// g > 0 (the next scale's factor, dividing f) u_next (+ bf16 shadow) =
// pool(resid, g) in the same pass.
cudaError_t launch_scale_advance(const int32_t* codes, const uint16_t* codebooks, int L, float* resid, float* q_out,
                                 float* u_next, uint16_t* u_next_bf16, int64_t rows_pooled, int64_t D, int64_t K, int f,
                                 int g, bool update_r, int* err, cudaStream_t stream);
// out[t] = bf16(sum_s q[s][t / f[s]]) in scale order.
cudaError_t launch_multiscale_recon(const float* const* q, const int* f, int S, uint16_t* out, int64_t rows, int64_t D,
                                    cudaStream_t stream);
cudaError_t launch_f32_to_bf16(const float* x, uint16_t* y, int64_t n, cudaStream_t stream);
cudaError_t launch_bf16_to_f32(const uint16_t* x, float* y, int64_t n, cudaStream_t stream);

// ---- bf16 linear (gemm.cu)
// y[M,N] = bf16(x[M,K] . w[N,K]^T + bias). If y_f32 is non-null the f32
// accumulator (+bias) is written there instead of the bf16 output.
int linear_bf16(ncm_ctx* ctx, const uint16_t* x, const uint16_t* w, const uint16_t* bias, uint16_t* y, float* y_f32,
                int64_t M, int64_t K, int64_t N, cudaStream_t stream);
// Epilogue variants of the same GEMM. mode 1: SwiGLU — w is [2F, K] (gate rows,
// then up rows), y [M, F] = bf16(bf16(silu(bf16(g))) * bf16(u)); needs M > 64
// and F % 128 == 0. mode 2: residual — y [M, N] is read and overwritten with
// bf16(y + bf16(x.w^T + bias)).
int linear_bf16_ex(ncm_ctx* ctx, const uint16_t* x, const uint16_t* w, const uint16_t* bias, uint16_t* y,
                   float* y_f32, int64_t M, int64_t K, int64_t N, cudaStream_t stream, int mode, int64_t F);

// ---- NCCL (comm.cu, loaded on first use)
// One all-gather of `count` elements of `bytes_per_elem` bytes from every
// rank: recv[r * count ..] = rank r's send. Items run as one NCCL group.
struct AllGatherItem {
  const void* send;
  void* recv;
  size_t count;
  int bytes_per_elem;
};
int comm_all_gather(ncm_ctx* ctx, const AllGatherItem* items, int n, cudaStream_t stream);
void comm_release(ncm_ctx* ctx);

// Fused QKV projection for M > 64: qkv [M, N] = bf16(x . w^T + bias) with
// rotate_head (bf16 mode) applied to every 64-column head below voff using
// the per-token bf16-rounded tables cos_bf/sin_bf [M, 64] (16-byte aligned),
// and the V columns (n >= voff) also written transposed to vt [(N - voff), M].
// N and voff multiples of 64.
int linear_qkv_rope(ncm_ctx* ctx, const uint16_t* x, const uint16_t* w, const uint16_t* bias, uint16_t* qkv,
                    uint16_t* vt, const uint16_t* cos_bf, const uint16_t* sin_bf, int64_t M, int64_t K, int64_t N,
                    int64_t voff, cudaStream_t stream);

// ---- codebook-tied head (head.cu, gemm.cu)
// logits [T, K] f32 = fmaf(2 s, z.E^T, -c) with c [K] = s esq - bias, z [T, d]
// and E [K, d] bf16; scal = {d_scale, exp(log_inv_T), -2 s} in device memory
// (s = exp(log_inv_T) / d_scale).
int tied_head_logits_gemm(ncm_ctx* ctx, const uint16_t* z, const uint16_t* codebook, const float* c,
                          const float* scal, float* logits, int64_t T, int64_t d, int64_t K, cudaStream_t stream);

// ---- kernel-3 convolution over row segments (conv.cu, gemm.cu)
//
// Rows are grouped into independent segments (batch items, NCM levels); the
// convolution zero-pads each segment on both ends. The GEMM reads a bf16 copy
// of the input in "padded" row order: one zero row before every segment and
// one after the last, so segment s (real rows [r_s, r_s + n_s)) occupies
// padded rows [r_s + s + 1, r_s + s + 1 + n_s), and the rows a tap reads past
// a segment's end are zeros. Columns are padded with zeros to a multiple of 64.
constexpr int kMaxConvSegments = 64;
struct SegMap {
  int seg_len;  // > 0: every segment has seg_len rows (the tables are unused)
  int nseg;
  int rstart[kMaxConvSegments + 1];  // real first row of each segment; rstart[nseg] = rows
  // padded row -> real row, or -1 for a pad row (or past the end)
  __host__ __device__ __forceinline__ long long real_row(long long p) const {
    if (seg_len > 0) {
      if (p < 1) return -1;
      const long long s = (p - 1) / (seg_len + 1);
      const long long off = p - 1 - s * (seg_len + 1);
      if (s >= nseg || off >= seg_len) return -1;
      return s * seg_len + off;
    }
    for (int s = 0; s < nseg; ++s) {
      const long long ps = rstart[s] + s + 1;
      if (p >= ps && p < ps + (rstart[s + 1] - rstart[s])) return rstart[s] + (p - ps);
    }
    return -1;
  }
  __host__ __device__ __forceinline__ long long padded_rows() const {
    return seg_len > 0 ? static_cast<long long>(nseg) * (seg_len + 1) + 1 : rstart[nseg] + nseg + 1;
  }
};
// Builds the map for `nseg` segments of the given lengths (nullptr: one
// segment of `rows`); uniform lengths use the closed form. false if too many.
bool make_segmap(SegMap* m, int64_t rows, int nseg, const int64_t* lengths);

// The GEMM's epilogue: val = alpha * X + beta * (acc + bias) with X the f32
// (or bf16) input row, then any of: out_f32 = val, out_bf16 = bf16(val),
// resid -= val, acc_f32 += val. All [rows, width] in real row order.
struct ConvEpilogue {
  const float* x_f32;
  const uint16_t* x_bf16;
  float* out_f32;
  uint16_t* out_bf16;
  float* resid;
  float* acc_f32;
  const float* bias;  // [width] f32 or null
  float alpha, beta;
};
// a_pad: [padded rows, dp] bf16 (the padded copy), w_pack: [width, 3*dp] bf16
// (tap-major repack of a [width, width, 3] kernel).
int conv3_gemm(ncm_ctx* ctx, const uint16_t* a_pad, const uint16_t* w_pack, const SegMap& map, int64_t dp,
               int64_t width, const ConvEpilogue& ep, cudaStream_t stream);
// [width_out, width_in, 3] kernel (bf16 bits or f32 values) -> [width_out, 3, dp] bf16, zero-padded.
cudaError_t launch_conv_repack(const uint16_t* w_bf16, const float* w_f32, uint16_t* out, int64_t width, int64_t dp,
                               cudaStream_t stream);
// x [rows, width] (f32 or bf16) -> padded bf16 copy [map.padded_rows(), dp].
cudaError_t launch_conv_pad(const float* x_f32, const uint16_t* x_bf16, uint16_t* out, const SegMap& map,
                            int64_t width, int64_t dp, cudaStream_t stream);
// Upsampling along time of q [B, Tq, D] to T = Tq * f rows per item
// (F.interpolate(size=T); mode 0 nearest, 1 linear with align_corners=False):
// Q -> out_f32 (nullable), bf16(Q) -> out_pad (the conv's padded copy with
// segments of T rows, nullable), resid -= Q and acc += Q (nullable).
cudaError_t launch_upsample(const float* q, int64_t B, int64_t Tq, int64_t T, int64_t D, int mode, float* out_f32,
                            uint16_t* out_pad, int64_t dp, float* resid, float* acc, cudaStream_t stream);

}  // namespace ncm
