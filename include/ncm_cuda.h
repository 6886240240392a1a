/*
 * ncm_cuda.h — C ABI of the ncmorph_b200 CUDA library (libncm_cuda.so).
 *
 * This is the drop-in boundary between ncmorph's host code (the Zig
 * `src/decoder.zig`, `src/ncm_body.zig`, `src/ncm_model.zig` callers and the
 * planned `packages/vq`) and hand-written sm_100a kernels. Each entry point
 * names the reference function it stands in for.
 *
 * Conventions
 *  - Every function returns NCM_OK (0) or a negative ncm status; none aborts,
 *    traps or prints. ncm_last_error() gives the message of the calling
 *    thread's last failure.
 *  - Pointers are DEVICE pointers unless the name ends in `_host_f32`, whose
 *    buffers are host memory in the reference's "f32 slice carrying bf16
 *    values" convention (src/loader.zig:338-341).
 *  - bf16 tensors are passed as uint16_t bit patterns, row-major.
 *  - Buffers are caller-owned. The context owns its device workspace.
 *  - Work is enqueued on `stream` (a cudaStream_t; NULL = legacy default
 *    stream) and is asynchronous, except the `_host_f32` functions, which
 *    return after the result is in host memory. ncm_sync() waits and also
 *    reports device-side failures (a timed-out pipeline wait, a bad index).
 *  - Shapes are validated on the host; a bad shape returns NCM_EINVAL where
 *    the reference would `std.debug.assert`.
 *  - A context may be used from one host thread at a time; different
 *    contexts (one per GPU, say) may be driven from different threads at
 *    once. The library's process-wide state (per-device kernel attributes
 *    and occupancy caches, the no-allocation scratch set-up) is atomic or
 *    locked.
 */
#ifndef NCM_CUDA_H
#define NCM_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define NCM_API __attribute__((visibility("default")))
#else
#define NCM_API
#endif

typedef struct ncm_ctx ncm_ctx_t;
typedef void* ncm_stream_t; /* cudaStream_t */

enum ncm_status {
  NCM_OK = 0,
  NCM_EINVAL = -1,   /* bad shape, null pointer or misaligned buffer */
  NCM_ECUDA = -2,    /* CUDA runtime error */
  NCM_ENOMEM = -3,   /* device workspace could not be allocated */
  NCM_ETIMEOUT = -4, /* a device-side bounded wait gave up */
  NCM_ERANGE = -5,   /* an index (token id, code) is out of range */
  NCM_ENOTSUP = -6   /* the device is not an sm_100 part */
};

/* ------------------------------------------------------------ context */

/* Creates a context on CUDA device `device` (must be compute capability 10.0).
 * Replaces the reference's implicit single-threaded CPU state: its kernels
 * take plain slices and keep nothing between calls
 * (packages/kernels/root.zig:96-104). The context holds the device, its
 * workspace, the device error word and, once bound, the NCCL communicator;
 * ncm_ctx_destroy, ncm_sync and the status and version queries after it have
 * no reference counterpart of their own. */
NCM_API int ncm_ctx_create(int device, ncm_ctx_t** out);
NCM_API int ncm_ctx_destroy(ncm_ctx_t* ctx);
/* Waits for `stream`, then checks the context's device error word. */
NCM_API int ncm_sync(ncm_ctx_t* ctx, ncm_stream_t stream);
NCM_API const char* ncm_status_string(int status);
NCM_API const char* ncm_last_error(void);
NCM_API int ncm_version(void);

/* --------------------------------------------------------- L7: bf16 */

/* y[i] = bf16(x[i]) with round-to-nearest-even and NaN -> 0x7FC0.
 * Replaces bf16_t.from_f32 (packages/bf16/root.zig:17-22) applied elementwise. */
NCM_API int ncm_f32_to_bf16(ncm_ctx_t* ctx, const float* x, uint16_t* y, int64_t n, ncm_stream_t stream);
/* y[i] = f32(x[i]) exactly. Replaces bf16_t.to_f32 / widen_little_endian
 * (packages/bf16/root.zig:25-37). */
NCM_API int ncm_bf16_to_f32(ncm_ctx_t* ctx, const uint16_t* x, float* y, int64_t n, ncm_stream_t stream);

/* ------------------------------------------------------ L1: bf16 linear */

/* y[M,N] = bf16( x[M,K] . W[N,K]^T (+ bias[N]) ), bf16 operands, f32
 * accumulation in tensor memory, one bf16 rounding at the output.
 * Replaces matmul_bf16 / matmul_bf16_bias (packages/kernels/root.zig:96-104,
 * matmul_bf16_impl :106-142). `bias` may be NULL. K must be a multiple of 8. */
NCM_API int ncm_linear_bf16(ncm_ctx_t* ctx, const uint16_t* x, const uint16_t* w, const uint16_t* bias, uint16_t* y,
                    int64_t M, int64_t K, int64_t N, ncm_stream_t stream);

/* Host-slice form of ncm_linear_bf16 with the reference's calling convention:
 * f32 slices whose values are rounded to bf16 on entry (as matmul_bf16_impl
 * does, root.zig:121-129) and an f32 output slice holding bf16 values.
 * Drop-in for kernels.matmul_bf16(_bias) (packages/kernels/root.zig:96-104). */
NCM_API int ncm_linear_bf16_host_f32(ncm_ctx_t* ctx, const float* x, const float* w, const float* bias, float* y,
                             int64_t M, int64_t K, int64_t N);

/* Host-slice stand-in for the f32 kernels.matmul (packages/kernels/root.zig:25-65)
 * used by ncm_body/ncm_model. It runs on the same bf16 tensor-core path
 * (operands rounded to bf16, f32 accumulation) and returns the f32
 * accumulator without the final bf16 rounding. */
NCM_API int ncm_matmul_host_f32(ncm_ctx_t* ctx, const float* x, const float* w, float* y, int64_t M, int64_t K,
                        int64_t N);

/* ------------------------------------------------- R1-R6: RVQ tokenizer */

/* sqnorm[k] = sum_d e[k,d]^2, accumulated in f64 and rounded once to f32.
 * The ||e_k||^2 term of the distance in research/reference/vq_forward_semantics.md:81. */
NCM_API int ncm_code_sqnorm(ncm_ctx_t* ctx, const uint16_t* codebook, float* sqnorm, int64_t K, int64_t D,
                    ncm_stream_t stream);

/* One residual-VQ level (vq_forward_semantics.md:68-72):
 *   codes[n] = argmin_k ( sqnorm[k] - 2 * bf16(residual[n]) . e[k] )  (lowest k on ties)
 *   residual[n] -= e[codes[n]]                                         (f32)
 * The distance GEMM runs on tcgen05 with bf16 operands and f32 accumulation.
 * residual [N,D] f32 in/out, codebook [K,D] bf16, sqnorm [K] f32 (NULL: computed),
 * codes [N] int32 out. D must be a multiple of 8. */
NCM_API int ncm_rvq_level(ncm_ctx_t* ctx, float* residual, const uint16_t* codebook, const float* sqnorm,
                  int32_t* codes, int64_t N, int64_t D, int64_t K, ncm_stream_t stream);

/* ncm_rvq_level that also reports each row's top-2 distance gap (the near-tie
 * measure of the parity rule; vq_forward_semantics.md:81):
 *   top2_gap[n] = (d2 - d1) / (||bf16(r_n)||^2 + d1)
 * where d1 <= d2 are the two smallest GEMM distances sqnorm[k] - 2 bf16(r_n) . e_k
 * of row n (so ||bf16(r_n)||^2 + d1 is the best full squared distance). Codes
 * and the residual update equal ncm_rvq_level's. top2_gap [N] f32 device. */
NCM_API int ncm_rvq_level_top2(ncm_ctx_t* ctx, float* residual, const uint16_t* codebook, const float* sqnorm,
                               int32_t* codes, float* top2_gap, int64_t N, int64_t D, int64_t K, ncm_stream_t stream);

/* L residual levels over x (vq_forward_semantics.md:59-82 at a single scale):
 * residual = f32(x); for l: ncm_rvq_level(codebooks[l]).
 * x [N,D] bf16; codebooks [L,K,D] bf16; sqnorms [L,K] f32 or NULL (computed);
 * codes [L,N] int32 out; recon [N,D] bf16 out or NULL (= decode of the codes);
 * residual_out [N,D] f32 out or NULL (the residual after the last level). */
NCM_API int ncm_rvq_encode(ncm_ctx_t* ctx, const uint16_t* x, const uint16_t* codebooks, const float* sqnorms, int32_t L,
                   int32_t* codes, uint16_t* recon, float* residual_out, int64_t N, int64_t D, int64_t K,
                   ncm_stream_t stream);

/* Host-buffer form of ncm_rvq_encode, as a host caller with plain slices
 * (the planned packages/vq) calls it: x_host [N,D] bf16 and codes_host [L,N],
 * recon_host [N,D] (nullable) are HOST memory; codebooks/sqnorms are device
 * buffers. Rows move in chunks so the host->device copies, the encode and the
 * device->host copies of neighbouring chunks overlap (page-locked host memory
 * gives full copy speed). Returns when the results are in host memory. */
NCM_API int ncm_rvq_encode_host(ncm_ctx_t* ctx, const uint16_t* x_host, const uint16_t* codebooks,
                                const float* sqnorms, int32_t L, int32_t* codes_host, uint16_t* recon_host,
                                int64_t N, int64_t D, int64_t K, ncm_stream_t stream);

/* ------------------------------------------- (e) row-sharded encode */

/* Token rows shard across GPUs with the codebooks replicated; the only
 * exchange is an NCCL all-gather of codes and reconstructions over NVLink.
 * No counterpart in the reference, which runs on one CPU thread and has no
 * distributed mode (PROJECT.md:35); each rank's rows follow
 * vq_forward_semantics.md:59-82 exactly as ncm_rvq_encode does.
 * One context per GPU (one process or thread each). ncm_comm_unique_id
 * fills 128 bytes on one rank, the caller ships them to every rank, and each
 * rank calls ncm_ctx_comm_init (collective; the context owns the
 * communicator and frees it in ncm_ctx_destroy). NCCL (libnccl.so.2) is
 * loaded on first use; NCM_ENOTSUP when it cannot be. */
NCM_API int ncm_comm_unique_id(uint8_t* id_out /* [128] */);
NCM_API int ncm_ctx_comm_init(ncm_ctx_t* ctx, const uint8_t* id /* [128] */, int32_t rank, int32_t nranks);

/* Rank r holds rows [r*n_local, (r+1)*n_local) of an N = nranks * n_local row
 * problem (pad N to a multiple of nranks). Each rank encodes its rows as
 * ncm_rvq_encode does and all-gathers: on return (stream-ordered) every rank
 * holds codes_all [L, N] int32 and, when recon_all is non-NULL, recon_all
 * [N, D] bf16. Collective: every rank calls it with the same L, n_local, D, K. */
NCM_API int ncm_rvq_encode_sharded(ncm_ctx_t* ctx, const uint16_t* x_local, const uint16_t* codebooks,
                                   const float* sqnorms, int32_t L, int32_t* codes_all, uint16_t* recon_all,
                                   int64_t n_local, int64_t D, int64_t K, ncm_stream_t stream);

/* Peer copies for the same exchange without SMs. No counterpart in the
 * reference (single CPU thread, no distributed mode). One process per GPU on
 * one node: a rank exports the IPC handle of a device buffer it allocated
 * with cudaMalloc (ncm_ipc_export records the buffer's offset inside its
 * allocation), ships the handle to the other ranks, and each maps it with
 * ncm_ipc_open, which returns the buffer's address in that process (unmap
 * with ncm_ipc_close). ncm_copy_async and ncm_copy2d_async are
 * cudaMemcpyAsync / cudaMemcpy2DAsync device-to-device on `stream`: with a
 * peer's mapping as source or destination they run on the copy engines over
 * NVLink, so the exchange takes no SM from kernels running meanwhile.
 * Ordering between ranks is the caller's: a copy into a peer's buffer must
 * start after the peer is done with it, and the peer may read it only after
 * the copy completed (a collective barrier on both sides serves). */
typedef struct ncm_ipc_handle {
  uint8_t handle[64]; /* cudaIpcMemHandle_t of the allocation */
  uint64_t offset;    /* the buffer's offset inside that allocation */
  uint64_t bytes;     /* the buffer's size */
} ncm_ipc_handle_t;
NCM_API int ncm_ipc_export(const void* dev_ptr, uint64_t bytes, ncm_ipc_handle_t* out);
NCM_API int ncm_ipc_open(const ncm_ipc_handle_t* handle, void** dev_ptr_out);
NCM_API int ncm_ipc_close(void* dev_ptr);
NCM_API int ncm_copy_async(void* dst, const void* src, uint64_t bytes, ncm_stream_t stream);
NCM_API int ncm_copy2d_async(void* dst, uint64_t dst_pitch, const void* src, uint64_t src_pitch,
                             uint64_t width_bytes, uint64_t rows, ncm_stream_t stream);

/* Area pooling by an integer factor (F.interpolate mode="area" with T % factor == 0,
 * vq_forward_semantics.md:67,80): y[b,j,:] = (sum_{i<factor} x[b,j*factor+i,:]) / factor,
 * summed in increasing i in f32. x [B,T,D] f32, y [B,T/factor,D] f32. */
NCM_API int ncm_pool_avg(ncm_ctx_t* ctx, const float* x, float* y, int64_t B, int64_t T, int64_t D, int32_t factor,
                 ncm_stream_t stream);

/* Decode (vq_forward_semantics.md:69,82): recon[n,:] = bf16( sum_l e_l[codes[l,n],:] ),
 * summed over l in increasing order in f32. codes [L,N]; codebooks [L,K,D]. A code
 * outside [0,K) makes the call fail with NCM_ERANGE (reported by ncm_sync); the rows
 * holding one are left unwritten, every other row is decoded. */
NCM_API int ncm_rvq_decode(ncm_ctx_t* ctx, const int32_t* codes, const uint16_t* codebooks, int32_t L, uint16_t* recon,
                   int64_t N, int64_t D, int64_t K, ncm_stream_t stream);

/* Upsampling along time, F.interpolate(size=out_len) on [B, C, T] data as the
 * quantiser's U_i (research/reference/vq_forward_semantics.md:82, :108):
 * q [batch, in_len, width] f32 -> out [batch, out_len, width] f32.
 * mode 0 nearest: src = min(floor(t * s), in_len - 1);
 * mode 1 linear (align_corners=False): src = max(fma(s, t + 0.5, -0.5), 0),
 *   i0 = trunc(src), l1 = src - i0, i1 = min(i0 + 1, in_len - 1),
 *   out = fma(q[i0], 1 - l1, q[i1] * l1)   (PyTorch's CPU operation order);
 * s = float(in_len) / float(out_len). width % 4 == 0. */
NCM_API int ncm_upsample(ncm_ctx_t* ctx, const float* q, float* out, int64_t batch, int64_t in_len, int64_t out_len,
                         int64_t width, int32_t mode, ncm_stream_t stream);

/* Kernel-3, padding-1 convolution along rows with a blend, per segment of
 * rows (each segment zero-padded on both ends; segment_lengths is a HOST
 * array of num_segments entries summing to rows, NULL = one segment):
 *   out[t,o] = alpha * x[t,o] + beta * (bias[o] + sum_{i,k} w[o,i,k] * x[t+k-1,i])
 * alpha = beta = 1 is apply_post_upsample_conv (src/ncm_model.zig:296-326);
 * alpha = 1 - r, beta = r is the quantiser's Phi (vq_forward_semantics.md:93-100).
 * x, out [rows, width] f32 (out may be x); weight [width, width, 3] bf16 (the
 * PyTorch Conv1d layout); bias [width] f32 or NULL. The sum runs on tcgen05
 * with bf16(x) and bf16 weights, f32 accumulation. Unequal segment lengths
 * allow at most 64 segments. */
NCM_API int ncm_conv1d_k3(ncm_ctx_t* ctx, const float* x, const uint16_t* weight, const float* bias, float* out,
                          int64_t rows, int64_t width, int32_t num_segments, const int64_t* segment_lengths,
                          float alpha, float beta, ncm_stream_t stream);

/* Host-slice form of ncm_model.apply_post_upsample_conv (src/ncm_model.zig:296-326):
 * input [row_count, width] f32 HOST, updated in place to input + bias + conv(input);
 * weight [width, width, 3] and bias [width] f32 HOST (bf16-representable values,
 * as loaded checkpoints are). Synchronous. */
NCM_API int ncm_post_upsample_conv_host_f32(ncm_ctx_t* ctx, float* input, const float* weight, const float* bias,
                                            int64_t row_count, int64_t width);

/* Multiscale tokenizer forward (research/ncm_facts.md:81; scales coarse -> fine):
 *   h = linear_bf16(x, w_in, b_in); r = f32(h); recon = 0
 *   for s: u = pool(r, f_s); L levels of ncm_rvq_level on u; q = sum_l e_{s,l}[code]
 *          Q = up(q, T) (upsample_mode); with Phi weights Q = Phi_s(Q)
 *          r -= Q; recon += Q                        (f32, scales in order)
 *   y = linear_bf16(bf16(recon), w_out, b_out)
 * Phi_s(Q) = (1 - phi_ratio) * Q + phi_ratio * (phi_bias[s] + Conv1d_k3(Q; phi_weight[s]))
 * per batch item (vq_forward_semantics.md:93-100, R_k = Phi o Up), computed as
 * ncm_conv1d_k3 does. Codes are written scale-major: scale s occupies
 * L * B*T/f_s entries, level-major. */
typedef struct ncm_tokenizer_config {
  int64_t batch;            /* B */
  int64_t seq_len;          /* T */
  int64_t model_width;      /* width of x and y */
  int64_t vq_width;         /* D, the quantised width */
  int64_t codebook_size;    /* K */
  int32_t num_scales;       /* S (<= 16) */
  int32_t levels_per_scale; /* L */
  int32_t pool_factors[16]; /* f_s, coarse to fine; each divides seq_len */
  int32_t upsample_mode;    /* 0 nearest repeat (default), 1 linear (ncm_upsample) */
  float phi_ratio;          /* r of Phi; used only when Phi weights are passed */
} ncm_tokenizer_config_t;

NCM_API int ncm_tokenizer_forward(ncm_ctx_t* ctx, const ncm_tokenizer_config_t* cfg, const uint16_t* x, const uint16_t* w_in,
                          const uint16_t* b_in, const uint16_t* codebooks, const float* sqnorms,
                          const uint16_t* w_out, const uint16_t* b_out, int32_t* codes, uint16_t* recon,
                          uint16_t* y, ncm_stream_t stream);

/* ncm_tokenizer_forward with the quantiser's residual convolutions:
 * phi_weight [S, D, D, 3] bf16 and phi_bias [S, D] f32 (both NULL: no Phi). */
NCM_API int ncm_tokenizer_forward_ex(ncm_ctx_t* ctx, const ncm_tokenizer_config_t* cfg, const uint16_t* x,
                                     const uint16_t* w_in, const uint16_t* b_in, const uint16_t* codebooks,
                                     const float* sqnorms, const uint16_t* phi_weight, const float* phi_bias,
                                     const uint16_t* w_out, const uint16_t* b_out, int32_t* codes, uint16_t* recon,
                                     uint16_t* y, ncm_stream_t stream);

/* Multiscale decode (R5 at every scale; vq_forward_semantics.md:70, :82):
 * recon [B, T, D] = bf16( sum_s Phi_s(up(q_s, T)) ) from codes laid out as
 * ncm_tokenizer_forward writes them; cfg->model_width is unused. Given the
 * tokenizer's codes, this reproduces its recon bit for bit. */
NCM_API int ncm_multiscale_decode(ncm_ctx_t* ctx, const ncm_tokenizer_config_t* cfg, const int32_t* codes,
                                  const uint16_t* codebooks, const uint16_t* phi_weight, const float* phi_bias,
                                  uint16_t* recon, ncm_stream_t stream);

/* ---------------------------- quantiser pieces around the RVQ levels */

/* Pre-quantisation GroupNorm, affine=False (research/reference/
 * vq_forward_semantics.md:43-49): x, y [batch, T, C] f32 (channels
 * contiguous); per sample and group of C/groups channels, statistics over all
 * T positions; y = (x - mean) / sqrt(var + eps), biased variance. */
NCM_API int ncm_group_norm(ncm_ctx_t* ctx, const float* x, float* y, int64_t batch, int64_t T, int64_t C,
                           int32_t groups, float eps, ncm_stream_t stream);

/* One stage of the learned level-0 cascade (vq_forward_semantics.md:127-139):
 * down: Conv1d(C, C, kernel 4, stride 4) over time, x [batch, L, C] ->
 * y [batch, L/4, C]; weight [C, C, 4] bf16 (Conv1d layout), bias [C] or NULL.
 * up: ConvTranspose1d(C, C, kernel 4, stride 4), x [batch, L, C] ->
 * y [batch, 4L, C]; weight [C_in, C_out, 4] bf16 (ConvTranspose1d layout).
 * Both run as one tcgen05 GEMM (bf16 operands, f32 accumulation, bf16 out). */
NCM_API int ncm_conv_down4(ncm_ctx_t* ctx, const uint16_t* x, const uint16_t* weight, const uint16_t* bias,
                           uint16_t* y, int64_t batch, int64_t L, int64_t C, ncm_stream_t stream);
NCM_API int ncm_conv_up4(ncm_ctx_t* ctx, const uint16_t* x, const uint16_t* weight, const uint16_t* bias,
                         uint16_t* y, int64_t batch, int64_t L, int64_t C, ncm_stream_t stream);

/* Codebook EMA of one level (vq_forward_semantics.md:141-173), in two steps
 * so a multi-GPU caller can sum the statistics across ranks in between:
 * stats: counts[k] = rows whose code is k, sums[k, :] = sum of those rows of
 *   u [N, D] f32 (in increasing row order: the same result on every run);
 * update: N <- decay N + (1 - decay) counts; n = sum N;
 *   N_hat = (N + eps) / (n + K eps) * n; m <- decay m + (1 - decay) sums;
 *   e = m / N_hat into codebook_f32 and/or codebook_bf16 (either NULL).
 * ema_count [K] and ema_sum [K, D] f32 are the persistent EMA buffers. */
NCM_API int ncm_ema_code_stats(ncm_ctx_t* ctx, const float* u, const int32_t* codes, float* counts, float* sums,
                               int64_t N, int64_t D, int64_t K, ncm_stream_t stream);
NCM_API int ncm_ema_update(ncm_ctx_t* ctx, const float* counts, const float* sums, float* ema_count, float* ema_sum,
                           float* codebook_f32, uint16_t* codebook_bf16, int64_t K, int64_t D, float decay,
                           float eps, ncm_stream_t stream);

/* ------------------------------------------------- checkpoint loading */

/* safetensors element types the loader reads (packages/safetensors/root.zig:34-54) */
enum { NCM_DTYPE_BF16 = 0, NCM_DTYPE_F16 = 1, NCM_DTYPE_F32 = 2 };

/* One tensor of a safetensors file to device memory as bf16 (src/loader.zig:
 * 286-345 read_tensor/decode_chunk, without widening to f32): nbytes at
 * absolute file offset `offset` (= 8 + header_len + data_offsets[0], from the
 * caller's parse_header) stream through pinned staging buffers to dst
 * (nbytes / element size bf16 values). BF16 is copied bit for bit; F16 and F32
 * round to bf16 on the device (nearest even, NaN -> 0x7FC0). Returns when the
 * data is on the device. */
NCM_API int ncm_load_tensor_bf16(ncm_ctx_t* ctx, const char* path, uint64_t offset, uint64_t nbytes, int32_t dtype,
                                 uint16_t* dst, ncm_stream_t stream);

/* ------------------------------------------- codebook-tied output head */

/* _TiedCodebookHead (PROJECT.md:222, decision D18): per predicted level,
 *   logits[t,k] = (2 z_t . E_k - E_sq[k]) / d_scale * exp(log_inv_T) + bias[k]
 * with E_sq[k] = sum_d E[k,d]^2 and d_scale = mean_k E_sq[k]. z [T, d] bf16 (the
 * head's Linear(n_embd -> d) output, e.g. from ncm_linear_bf16), codebook E
 * [K, d] bf16, esq [K] f32 or NULL (computed), bias [K] f32 or NULL. The dot
 * products run on tcgen05 (bf16 operands, f32 accumulation). d % 8 == 0. */
NCM_API int ncm_tied_head_logits(ncm_ctx_t* ctx, const uint16_t* z, const uint16_t* codebook, const float* esq,
                                 const float* bias, float log_inv_T, float* logits, int64_t T, int64_t d, int64_t K,
                                 ncm_stream_t stream);

/* codes[t] = argmax_k logits[t,k] (lowest k among equal values), the
 * temperature-0 pick of _sample_level_raw, without materialising the logits:
 * the argmin runs in the distance GEMM's epilogue as in ncm_rvq_level. */
NCM_API int ncm_tied_head_argmax(ncm_ctx_t* ctx, const uint16_t* z, const uint16_t* codebook, const float* esq,
                                 const float* bias, float log_inv_T, int32_t* codes, int64_t T, int64_t d, int64_t K,
                                 ncm_stream_t stream);

/* -------------------------------------- L3-L6: NCM decoder forward pieces */

/* Row-wise bf16 RMSNorm: y = bf16(bf16(x * inv) * bf16(w)), inv = 1/sqrt(mean(x^2) + eps)
 * in f32, then + bias (rounded) when bias is non-NULL. x, y [rows, width] bf16 (width % 8 == 0).
 * Replaces kernels.rms_norm_bf16 (packages/kernels/root.zig:243-252) applied per row
 * (src/decoder.zig:234-251) and ncm_norm.rms_norm_rows_with_bias (src/ncm_norm.zig:21-49).
 * The sum of squares is a tree sum, not PyTorch's cascade (root.zig:152-224). */
NCM_API int ncm_rms_norm_bf16(ncm_ctx_t* ctx, const uint16_t* x, const uint16_t* w, const uint16_t* bias, uint16_t* y,
                              int64_t rows, int64_t width, float eps, ncm_stream_t stream);

/* out[t, :] = table[ids[t], :] (bf16). Replaces kernels.embedding_row
 * (packages/kernels/root.zig:288-301) over a sequence; an id outside [0, vocab)
 * makes ncm_sync report NCM_ERANGE (decoder.zig:107 returns TokenIdOutOfRange). */
NCM_API int ncm_embedding_gather(ncm_ctx_t* ctx, const uint16_t* table, int64_t vocab, int64_t width,
                                 const int32_t* ids, int64_t T, uint16_t* out, ncm_stream_t stream);

/* Host function: RoPE cos/sin tables [T, head_dim] at explicit positions, with
 * libm powf/cosf/sinf exactly as rope_default + rope_tables (root.zig:305-348)
 * and ncm_position.tables_at_positions (src/ncm_position.zig:71-118) build them. */
NCM_API int ncm_rope_tables_host(int32_t head_dim, float theta, const int32_t* positions, int64_t T, float* cos_out,
                                 float* sin_out);

/* Host function: the same tables from Llama 3 scaled frequencies, as
 * rope_llama3 (packages/kernels/root.zig:636-666) adjusts rope_default's
 * (factor, low/high frequency factors, original context length: the
 * rope_scaling of a Llama 3 config.json). Its assertions (:645-648) are
 * reported as NCM_EINVAL. */
NCM_API int ncm_rope_tables_llama3_host(int32_t head_dim, float theta, float factor, float low_freq_factor,
                                        float high_freq_factor, int64_t original_max_position_embeddings,
                                        const int32_t* positions, int64_t T, float* cos_out, float* sin_out);

/* Attention mask description. mode: 0 causal (causal_mask, root.zig:380-399;
 * ncm_model's source_causal, src/ncm_model.zig:199-203), 1 block-diagonal
 * (src/ncm_mask.zig:10-42), 2 block-causal (each level also sees every earlier
 * level). In block modes positions are [prefix | level 0 | level 1 | ...];
 * prefix_pad_mask bit i marks prefix key i as padding (prefix_length <= 64).
 * sliding_window (causal mode only; 0 = none): query q sees keys
 * q - sliding_window < k <= q. ncm_attention_bf16 ignores the levels in causal
 * mode; ncm_ncm_forward still takes its RoPE positions and level embeddings
 * from prefix_length and level_lengths there, as ncm_model does. */
typedef struct ncm_mask {
  int32_t mode;
  int32_t prefix_length;
  uint64_t prefix_pad_mask;
  int32_t num_levels;
  int32_t level_lengths[32];
  int32_t sliding_window;
} ncm_mask_t;

/* Multi-head GQA attention core of attention_impl in bf16 mode
 * (packages/kernels/root.zig:450-581) from projected rows: qkv [T, qkv_stride]
 * bf16 holds Q (heads*64 columns), then K (kv_heads*64), then V (kv_heads*64).
 * If cos/sin [T, 64] (device f32) are given, RoPE is applied IN PLACE to the
 * Q and K columns first (rotate_head bf16 mode, root.zig:615-633). out [T, heads*64]
 * bf16 is the context before the output projection. head_dim must be 64; T % 8 == 0. */
NCM_API int ncm_attention_bf16(ncm_ctx_t* ctx, uint16_t* qkv, int64_t qkv_stride, const float* cos_t,
                               const float* sin_t, uint16_t* out, int64_t T, int32_t heads, int32_t kv_heads,
                               const ncm_mask_t* mask, ncm_stream_t stream);

/* ncm_attention_bf16 for layers with QK-norm (attention_impl with
 * query_norm_weight and key_norm_weight, packages/kernels/root.zig:471,
 * :500-530, bf16 mode): every Q head of qkv gets rms_norm_bf16 (root.zig:
 * 243-252) with q_norm [64] and every K head with k_norm [64] (bf16 device,
 * both required), eps = the config's rms_norm_epsilon, then RoPE if cos/sin
 * are given, IN PLACE, before the attention. Bit-identical to the reference's
 * norm and rotation (its sum-of-squares order included). */
NCM_API int ncm_attention_qk_norm_bf16(ncm_ctx_t* ctx, uint16_t* qkv, int64_t qkv_stride, const float* cos_t,
                                       const float* sin_t, const uint16_t* q_norm, const uint16_t* k_norm, float eps,
                                       uint16_t* out, int64_t T, int32_t heads, int32_t kv_heads,
                                       const ncm_mask_t* mask, ncm_stream_t stream);

/* Fused QKV projection of one decoder layer (src/decoder.zig:171-190 and
 * rotate_head, packages/kernels/root.zig:615-633): qkv [T, (heads + 2 kv_heads) * 64]
 * = bf16(x . w^T + bias) with RoPE (bf16 mode, tables cos_t/sin_t [T, 64] f32
 * device) applied to the Q and K heads in the GEMM epilogue, and vt
 * [kv_heads * 64, T] receiving the V heads transposed (the attention's P.V
 * operand). Bit-identical to ncm_linear_bf16 followed by the RoPE that
 * ncm_attention_bf16 applies. head_dim 64; T > 64. */
NCM_API int ncm_qkv_projection_rope(ncm_ctx_t* ctx, const uint16_t* x, const uint16_t* w, const uint16_t* bias,
                                    const float* cos_t, const float* sin_t, uint16_t* qkv, uint16_t* vt, int64_t T,
                                    int64_t hidden, int32_t heads, int32_t kv_heads, ncm_stream_t stream);

/* NCM body forward (src/ncm_model.zig:89-250) with the bf16 layer of
 * src/decoder.zig:168-216: input projection (+bias), level embeddings,
 * per-level restarting RoPE positions, the configured mask, num_layers x
 * [RMSNorm, fused QKV, RoPE, attention, O projection, residual, RMSNorm,
 * fused gate|up, SiLU*up, down, residual], final RMSNorm (+bias). All
 * activations bf16, f32 accumulation. T = prefix_length + sum(level_lengths). */
typedef struct ncm_decoder_config {
  int64_t hidden_size;
  int64_t vq_width;
  int64_t num_attention_heads;
  int64_t num_key_value_heads;
  int64_t head_dim; /* must be 64 */
  int64_t intermediate_size;
  float rms_norm_epsilon;
  float rope_theta; /* RoPE base (rope_default's theta) */
  int32_t use_level_encoding;
  ncm_mask_t mask;
  /* RoPE frequencies: 0 rope_default, 1 rope_llama3 (root.zig:636-666) with
   * the four parameters below (ignored for 0) */
  int32_t rope_type;
  float rope_factor;
  float rope_low_freq_factor;
  float rope_high_freq_factor;
  int64_t rope_original_max_position_embeddings;
} ncm_decoder_config_t;

typedef struct ncm_decoder_layer_weights {
  const uint16_t* ln_1;      /* [hidden] */
  const uint16_t* qkv;       /* [(H + 2*Hkv)*64, hidden]: the fused_qkv_weight of ncm_model.zig:37 */
  const uint16_t* qkv_bias;  /* nullable */
  const uint16_t* o;         /* [hidden, H*64] */
  const uint16_t* o_bias;    /* nullable */
  const uint16_t* ln_2;      /* [hidden] */
  const uint16_t* gate_up;   /* [2*F, hidden]: gate_weight rows, then up_weight rows */
  const uint16_t* down;      /* [hidden, F] */
  /* QK-norm (ncm_model.zig:42-43, root.zig:500-530): per-head RMSNorm scales
   * [64] for the Q and K heads, applied before RoPE with rms_norm_epsilon;
   * both or NULL (Qwen3-style checkpoints carry them) */
  const uint16_t* q_norm;
  const uint16_t* k_norm;
} ncm_decoder_layer_weights_t;

typedef struct ncm_decoder_weights {
  const uint16_t* input_projection;      /* [hidden, vq_width] */
  const uint16_t* input_projection_bias; /* [hidden] */
  const uint16_t* level_embedding;       /* [num_levels, hidden] */
  const uint16_t* final_norm;            /* [hidden] */
  const uint16_t* final_norm_bias;       /* nullable */
  int32_t num_layers;
  const ncm_decoder_layer_weights_t* layers; /* host array of num_layers entries (device pointers) */
  /* post_upsample_convs (ncm_model.zig:71, :141-153), applied to each level's
   * input rows before the input projection: [num_levels, vq_width, vq_width, 3]
   * bf16 and [num_levels, vq_width] f32, or both NULL */
  const uint16_t* post_conv_weight;
  const float* post_conv_bias;
} ncm_decoder_weights_t;

/* inputs [T, vq_width] bf16: the assembled prefix + target rows (ncm_model.zig:128-140);
 * out [T, hidden] bf16: final-normalised hidden states in [prefix | levels] order. */
NCM_API int ncm_ncm_forward(ncm_ctx_t* ctx, const ncm_decoder_config_t* cfg, const ncm_decoder_weights_t* weights,
                            const uint16_t* inputs, uint16_t* out, ncm_stream_t stream);

/* No counterpart in the reference: ncmorph has no device code, so nothing
 * there allocates device memory. This is ncm_rvq_level for callers that
 * cannot call cudaMalloc: host plugins whose application owns every device
 * allocation (its arena or caching allocator must account for all memory),
 * and latency-bound paths that may not stall on cudaMalloc, which can
 * synchronise the device. It takes no context and allocates
 * nothing: its scratch (an error word, the bf16 copy of the residual, the
 * per-split argmin partials, the code norms when sqnorm is NULL) is a 16 MiB
 * device array that every GPU loading the library holds
 * until exit, so 2*N*D + 4*K bytes (plus split partials) must fit in it;
 * larger problems are rejected with NCM_EINVAL. It runs on the current
 * device, in the current CUDA context; the first call in each context looks
 * up the array's device address (make that call before any stream capture).
 * All calls share the array: calls that overlap on the GPU race. It runs
 * ncm_rvq_level's plan and kernels, so codes and residual equal that entry
 * point's bit for bit. Device-side failures (a bounded wait that gave up, an
 * out-of-range code) accumulate in the array's error word until
 * ncm_rvq_level_noalloc_status reads it. */
NCM_API int ncm_rvq_level_noalloc(float* residual, const uint16_t* codebook, const float* sqnorm, int32_t* codes,
                                  int64_t N, int64_t D, int64_t K, ncm_stream_t stream);

/* No counterpart in the reference (companion of ncm_rvq_level_noalloc, which
 * has no context to carry errors). Waits for `stream`, reads the error word of
 * the current context's no-allocation scratch into *flags (nullable; bit 1 a
 * wait timed out, bit 2 an out-of-range index), clears it, and returns NCM_OK,
 * NCM_ETIMEOUT or NCM_ERANGE accordingly. Allocates nothing. */
NCM_API int ncm_rvq_level_noalloc_status(ncm_stream_t stream, int32_t* flags);

/* ------------------------------------------------------- measurement */

/* Benchmark instrumentation (no reference counterpart: ncmorph has no timing
 * code). Launch counts per kernel family are always kept; while profiling is
 * enabled, CUDA events are also recorded on the launch stream around every
 * launch. ncm_profile_read synchronises, returns the summed device time (ms)
 * and launch count of one family since the last read, and resets them.
 * Families: "rvq_argmin", "rvq_apply", "linear_bf16", "rvq_decode",
 * "code_sqnorm", "pool_avg", "scale_update", "cast", "attention",
 * "decoder_elementwise", "conv_k3", "upsample"; "*" = all of them. */
NCM_API int ncm_profile_enable(ncm_ctx_t* ctx, int on);
NCM_API int ncm_profile_read(ncm_ctx_t* ctx, const char* kernel, double* total_ms, int64_t* launches);

#ifdef __cplusplus
}
#endif

#endif /* NCM_CUDA_H */
