// Fused masked GQA attention on tcgen05 (L3), for the NCM decoder forward.
//
// One CTA per (128-query tile, query head). Per key tile of 128:
//   S = Q . K^T           tcgen05.mma M=128 N=128 K=64, f32 in TMEM (2 buffers)
//   online softmax        4 epilogue warps, one query row per thread, in registers
//   P (bf16) -> smem      128-byte-swizzled, the A operand of the next MMA
//   O_tile = P . V        tcgen05.mma M=128 N=64 K=128, f32 in TMEM (2 buffers)
//   o = o*alpha + O_tile  accumulated in registers with the running-max correction
// The MMA of S for tile j+1 and of P.V for tile j overlap the softmax of the
// neighbouring tiles. Key tiles that the mask removes entirely are never
// loaded. K tiles come straight from the fused QKV projection output by TMA;
// V is read transposed ([kv_head*64 + d][t], written by the RoPE kernel) so
// both MMAs take K-major operands.
//
// Score rounding follows ncmorph's bf16 attention (packages/kernels/root.zig:
// 546-548): s = bf16(bf16(q.k) * scale). The softmax is computed online
// (running max), probabilities enter the P.V product as bf16, and the
// context is rounded once to bf16 — within the bf16 bar of the reference's
// materialised softmax, not bit-equal to it.
#include <cfloat>
#include <cmath>

#include "internal.h"
#include "ptx.cuh"

namespace ncm {
namespace {

constexpr int AT_Q = 128;       // queries per CTA
constexpr int AT_K = 128;       // keys per tile
constexpr int AT_D = 64;        // head dim (fixed)
constexpr int AT_STAGES = 3;
constexpr int AT_THREADS = 320;  // w0 TMA, w1 MMA, w2-9 softmax
constexpr uint32_t AT_TMEM_COLS = 512;  // S: 2 x 128 cols, O: 2 x 64 cols
constexpr int kMaxLevels = 32;

struct __align__(1024) AttnSmem {
  uint8_t q[AT_Q * AT_D * 2];                 // 16 KB
  uint8_t k[AT_STAGES][AT_K * AT_D * 2];      // 16 KB each
  uint8_t vt[AT_STAGES][2][AT_D * 64 * 2];    // 2 x 8 KB each: [64 d rows x 64 keys] per half
  uint8_t p[2][2][AT_Q * 64 * 2];             // 2 buffers x 2 key halves x 16 KB
  uint64_t q_full;
  uint64_t kv_full[AT_STAGES];
  uint64_t kv_empty[AT_STAGES];
  uint64_t s_full[2];
  uint64_t s_empty[2];
  uint64_t p_full[2];
  uint64_t p_empty[2];
  uint64_t o_full[2];
  uint64_t o_empty[2];
  uint64_t mx_ready[2];
  uint64_t l_ready;
  uint64_t drain;
  float mx[2][2][AT_Q];   // [tile parity][key half][row] partial row maxima
  float lsum[2][AT_Q];    // [key half][row] final partial row sums
  uint32_t tmem_base;
  int abort_flag;
};
constexpr size_t ATTN_SMEM = sizeof(AttnSmem) + 1024;
static_assert(ATTN_SMEM <= 232448, "attention smem budget");

struct AttnArgs {
  uint16_t* out;  // [T, H*64] bf16
  int* err;
  int T, H, Hkv;
  int mode;        // 0 causal, 1 block-diagonal, 2 block-causal
  int prefix;      // P (block modes)
  unsigned long long pad_mask;  // bit i set: prefix key i is padding
  int nlev;
  int level_start[kMaxLevels + 1];  // level i spans [level_start[i], level_start[i+1])
  float scale;
};

__device__ __forceinline__ int level_of(const AttnArgs& a, int pos) {
  int l = 0;
  while (l + 1 < a.nlev && pos >= a.level_start[l + 1]) ++l;
  return l;
}

// Key intervals the CTA's queries may see: [0, P) and [A, B).
__device__ __forceinline__ void cta_key_span(const AttnArgs& a, int q0, int& P, int& A, int& B) {
  const int qmax = min(q0 + AT_Q - 1, a.T - 1);
  if (a.mode == 0) {
    P = 0;
    A = 0;
    B = qmax + 1;
    return;
  }
  P = a.prefix;
  if (qmax < P) {
    A = B = P;
    return;
  }
  const int lmax = level_of(a, qmax);
  B = a.level_start[lmax + 1];
  if (a.mode == 2) {
    A = P;
  } else {
    A = a.level_start[level_of(a, max(q0, P))];
  }
}

__device__ __forceinline__ bool tile_needed(int t, int P, int A, int B) {
  const int k0 = t * AT_K;
  return k0 < P || (k0 < B && k0 + AT_K > A);
}

__device__ __forceinline__ bool key_allowed(int k, int P, int lo, int hi, unsigned long long pad_mask) {
  return k < P ? !((pad_mask >> k) & 1ull) : (k >= lo && k < hi);
}

__device__ __forceinline__ void raise_abort_attn(volatile int* abort_flag, int* err) {
  *abort_flag = 1;
  atomicOr(err, kErrWaitTimeout);
}

__global__ void __launch_bounds__(AT_THREADS, 1)
    attention_bf16_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmVt, const AttnArgs args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  AttnSmem& S = *reinterpret_cast<AttnSmem*>(smem_raw + pad);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = blockIdx.x * AT_Q;
  const int h = blockIdx.y;
  const int kvh = h / (args.H / args.Hkv);
  int P, A, B;
  cta_key_span(args, q0, P, A, B);
  const int n_tiles_all = (max(B, P) + AT_K - 1) / AT_K;

  if (threadIdx.x == 0) {
    mbar_init(&S.q_full, 1);
    for (int s = 0; s < AT_STAGES; ++s) {
      mbar_init(&S.kv_full[s], 1);
      mbar_init(&S.kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&S.s_full[b], 1);
      mbar_init(&S.s_empty[b], 8);
      mbar_init(&S.p_full[b], 8);
      mbar_init(&S.p_empty[b], 1);
      mbar_init(&S.o_full[b], 1);
      mbar_init(&S.o_empty[b], 8);
      mbar_init(&S.mx_ready[b], 8);
    }
    mbar_init(&S.l_ready, 8);
    mbar_init(&S.drain, 1);
    S.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&S.tmem_base, AT_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = S.tmem_base;
  volatile int* abort_flag = &S.abort_flag;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------ TMA producer
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmVt);
      mbar_arrive_expect_tx(&S.q_full, AT_Q * AT_D * 2);
      tma_load_2d(&tmQ, &S.q_full, S.q, h * AT_D, q0);
      int stage = 0;
      uint32_t phase = 0;
      bool issued[AT_STAGES];
      uint32_t iss_par[AT_STAGES];
      for (int s = 0; s < AT_STAGES; ++s) issued[s] = false, iss_par[s] = 0;
      bool ok = true;
      for (int t = 0; t < n_tiles_all && ok; ++t) {
        if (!tile_needed(t, P, A, B)) continue;
        if (!mbar_wait(&S.kv_empty[stage], phase ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&S.kv_full[stage], AT_K * AT_D * 2 + 2 * AT_D * 64 * 2);
        tma_load_2d(&tmK, &S.kv_full[stage], S.k[stage], kvh * AT_D, t * AT_K);
        tma_load_2d(&tmVt, &S.kv_full[stage], S.vt[stage][0], t * AT_K, kvh * AT_D);
        tma_load_2d(&tmVt, &S.kv_full[stage], S.vt[stage][1], t * AT_K + 64, kvh * AT_D);
        issued[stage] = true;
        iss_par[stage] = phase;
        if (++stage == AT_STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) {
        raise_abort_attn(abort_flag, args.err);
        mbar_wait(&S.q_full, 0, nullptr);
        for (int s = 0; s < AT_STAGES; ++s)
          if (issued[s]) mbar_wait(&S.kv_full[s], iss_par[s], nullptr);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------ MMA issuer
      const uint32_t idesc_s = idesc_bf16_f32(AT_Q, AT_K);
      const uint32_t idesc_o = idesc_bf16_f32(AT_Q, AT_D);
      bool ok = mbar_wait(&S.q_full, 0, abort_flag);
      tc_fence_after();
      const uint32_t qa = smem_u32(S.q);
      int stage = 0, prev_stage = 0;
      uint32_t phase = 0;
      int j = 0;  // index among needed tiles
      for (int t = 0; t <= n_tiles_all && ok; ++t) {
        const bool have = t < n_tiles_all && tile_needed(t, P, A, B);
        if (t < n_tiles_all && !have) continue;
        if (have) {
          // S_j = Q . K^T
          const uint32_t b = j & 1, bp = (j >> 1) & 1;
          if (!mbar_wait(&S.kv_full[stage], phase, abort_flag) || !mbar_wait(&S.s_empty[b], bp ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t ka = smem_u32(S.k[stage]);
#pragma unroll
          for (int k = 0; k < AT_D / 16; ++k)
            tc_mma_f16(tmem + b * AT_K, smem_desc_k_sw128(qa + k * 32), smem_desc_k_sw128(ka + k * 32), idesc_s,
                       k != 0 ? 1u : 0u);
          tc_commit(&S.s_full[b]);
        }
        if (j > 0) {
          // O_{j-1} = P_{j-1} . V_{j-1}
          const int jp = j - 1;
          const uint32_t b = jp & 1, bp = (jp >> 1) & 1;
          if (!mbar_wait(&S.p_full[b], bp, abort_flag) || !mbar_wait(&S.o_empty[b], bp ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < AT_K / 16; ++kk) {
            const uint32_t pa = smem_u32(S.p[b][kk >> 2]) + (kk & 3) * 32;
            const uint32_t va = smem_u32(S.vt[prev_stage][kk >> 2]) + (kk & 3) * 32;
            tc_mma_f16(tmem + 2 * AT_K + b * AT_D, smem_desc_k_sw128(pa), smem_desc_k_sw128(va), idesc_o,
                       kk != 0 ? 1u : 0u);
          }
          tc_commit(&S.o_full[b]);
          tc_commit(&S.p_empty[b]);
          tc_commit(&S.kv_empty[prev_stage]);
        }
        if (have) {
          prev_stage = stage;
          if (++stage == AT_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
          ++j;
        } else {
          break;
        }
      }
      if (!ok) {
        raise_abort_attn(abort_flag, args.err);
        tc_commit(&S.drain);
        mbar_wait(&S.drain, 0, nullptr);
      }
    }
  } else {
    // ------------------------------------------------- softmax / epilogue
    // Eight warps: warp w reads TMEM lanes 32*(w%4).. (its 32 query rows) and
    // owns key columns [64*hf, 64*hf + 64) of each S tile and output dims
    // [32*hf, 32*hf + 32) of O, hf = (w - 2) / 4. The two warps of a row group
    // swap their partial row maxima through shared memory each tile.
    // Scores live in the log2 domain: t = bf16(q.k) * scale * log2(e), so
    // p = 2^(t - max t) and alpha = 2^(old max - new max).
    const int qw = warp & 3;
    const int hf = (warp - 2) >> 2;
    const int row = qw * 32 + lane;
    const int q = q0 + row;
    int lo = 0, hi = 0;
    if (args.mode == 0) {
      lo = 0;
      hi = q + 1;
    } else if (q >= args.prefix && q < args.T) {
      const int lq = level_of(args, q);
      hi = args.level_start[lq + 1];
      lo = args.mode == 2 ? args.prefix : args.level_start[lq];
    }
    const int Pq = args.mode == 0 ? 0 : args.prefix;
    const float c_scale = args.scale * 1.4426950408889634f;
    constexpr int HK = AT_K / 2, HD = AT_D / 2;
    float o[HD];
#pragma unroll
    for (int d = 0; d < HD; ++d) o[d] = 0.f;
    float m = -INFINITY, l = 0.f, alpha_prev = 1.f;
    bool ok = true;
    int j = 0;
    for (int t = 0; t < n_tiles_all; ++t) {
      if (!tile_needed(t, P, A, B)) continue;
      const uint32_t b = j & 1, bp = (j >> 1) & 1;
      if (!mbar_wait(&S.s_full[b], bp, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t sbase = tmem + (static_cast<uint32_t>(qw * 32) << 16) + b * AT_K + hf * HK;
      const int k0 = t * AT_K + hf * HK;
      const bool unmasked = __all_sync(0xffffffffu, k0 >= Pq && k0 >= lo && k0 + HK <= hi);
      // pass 1: max of this warp's 64 raw scores per row (rounding to bf16 is
      // monotonic, so the max of the rounded scores is the rounded max); in a
      // tile the mask touches, disallowed scores become -inf in TMEM first
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < HK; c += 32) {
        uint32_t v[32];
        tmem_ld_x32(sbase + c, v);
        tmem_wait_ld();
        if (!unmasked) {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (!key_allowed(k0 + c + i, Pq, lo, hi, args.pad_mask)) v[i] = __float_as_uint(-INFINITY);
          tmem_st_x32(sbase + c, v);
        }
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          mx0 = fmaxf(mx0, __uint_as_float(v[i]));
          mx1 = fmaxf(mx1, __uint_as_float(v[i + 1]));
        }
      }
      if (!unmasked) tmem_wait_st();
      // swap partial maxima with the partner warp (same rows, other key half)
      S.mx[b][hf][row] = fmaxf(mx0, mx1);
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.mx_ready[b]);
      if (!mbar_wait(&S.mx_ready[b], bp, abort_flag)) {
        ok = false;
        break;
      }
      const float raw_max = fmaxf(S.mx[b][0][row], S.mx[b][1][row]);
      const float mt = bf16lo(cvt_bf16x2(raw_max, 0.f)) * c_scale;
      const float m_new = fmaxf(m, mt);
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = ex2_approx(m - m_use);  // m = -inf -> 0
      // P_j (bf16): this warp's key half goes to P block hf; wait until P.V_{j-2} released it
      if (!mbar_wait(&S.p_empty[b], bp ^ 1u, abort_flag)) {
        ok = false;
        break;
      }
      // pass 2: t = bf16(s) * scale*log2e - m, p = 2^t, packed f32x2 arithmetic
      const unsigned long long cs2 = f2_pack(c_scale, c_scale), nm2 = f2_pack(-m_use, -m_use);
      unsigned long long rs2 = f2_pack(0.f, 0.f);
      uint8_t* prow = S.p[b][hf] + row * 128;
#pragma unroll 1
      for (int c = 0; c < HK; c += 32) {
        uint32_t v[32];
        tmem_ld_x32(sbase + c, v);
        tmem_wait_ld();
        const int ch0 = c >> 3;
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {  // four 16-byte chunks of 8 keys
          uint32_t w4[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int i = q4 * 8 + e * 2;
            const uint32_t pr = cvt_bf16x2(__uint_as_float(v[i]), __uint_as_float(v[i + 1]));
            const unsigned long long t2 = f2_fma(f2_pack(bf16lo(pr), bf16hi(pr)), cs2, nm2);
            float t0, t1;
            f2_unpack(t2, t0, t1);
            const float p0 = ex2_approx(t0), p1 = ex2_approx(t1);
            w4[e] = cvt_bf16x2(p0, p1);
            rs2 = f2_add(rs2, f2_pack(p0, p1));
          }
          const int sw = (ch0 + q4) ^ (row & 7);  // 128-byte swizzle: 16-byte chunk XOR row%8
          *reinterpret_cast<uint4*>(prow + sw * 16) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
        }
      }
      float rs0, rs1;
      f2_unpack(rs2, rs0, rs1);
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&S.s_empty[b]);
        mbar_arrive(&S.p_full[b]);
      }
      l = l * alpha + (rs0 + rs1);  // this warp's half of the row sum
      m = m_new;
      // fold in this warp's 32 columns of O_{j-1}
      if (j > 0) {
        const uint32_t bo = (j - 1) & 1, bop = ((j - 1) >> 1) & 1;
        if (!mbar_wait(&S.o_full[bo], bop, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t v[HD];
        tmem_ld_x32(tmem + (static_cast<uint32_t>(qw * 32) << 16) + 2 * AT_K + bo * AT_D + hf * HD, v);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.o_empty[bo]);
        const unsigned long long ap2 = f2_pack(alpha_prev, alpha_prev);
#pragma unroll
        for (int i = 0; i < HD; i += 2) {
          const unsigned long long r2 =
              f2_fma(f2_pack(o[i], o[i + 1]), ap2, f2_pack(__uint_as_float(v[i]), __uint_as_float(v[i + 1])));
          f2_unpack(r2, o[i], o[i + 1]);
        }
      }
      alpha_prev = alpha;
      ++j;
    }
    if (ok && j > 0) {
      const uint32_t bo = (j - 1) & 1, bop = ((j - 1) >> 1) & 1;
      if (!mbar_wait(&S.o_full[bo], bop, abort_flag)) {
        ok = false;
      } else {
        tc_fence_after();
        uint32_t v[HD];
        tmem_ld_x32(tmem + (static_cast<uint32_t>(qw * 32) << 16) + 2 * AT_K + bo * AT_D + hf * HD, v);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.o_empty[bo]);
#pragma unroll
        for (int i = 0; i < HD; ++i) o[i] = fmaf(o[i], alpha_prev, __uint_as_float(v[i]));
      }
    }
    // the full row sum is the sum of both halves' sums
    if (ok) {
      S.lsum[hf][row] = l;
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.l_ready);
      ok = mbar_wait(&S.l_ready, 0, abort_flag);
    }
    if (!ok) raise_abort_attn(abort_flag, args.err);
    if (ok && q < args.T) {
      const float lt = S.lsum[0][row] + S.lsum[1][row];
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
      uint16_t* dst = args.out + static_cast<size_t>(q) * args.H * AT_D + h * AT_D + hf * HD;
#pragma unroll
      for (int c = 0; c < HD; c += 8) {
        uint4 w;
        w.x = cvt_bf16x2(o[c + 0] * inv, o[c + 1] * inv);
        w.y = cvt_bf16x2(o[c + 2] * inv, o[c + 3] * inv);
        w.z = cvt_bf16x2(o[c + 4] * inv, o[c + 5] * inv);
        w.w = cvt_bf16x2(o[c + 6] * inv, o[c + 7] * inv);
        *reinterpret_cast<uint4*>(dst + c) = w;
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, AT_TMEM_COLS);
  }
}

}  // namespace

int attention_bf16(ncm_ctx* ctx, const uint16_t* qkv, int64_t qkv_stride, const uint16_t* vt, uint16_t* out, int T,
                   int H, int Hkv, int mode, int prefix, unsigned long long pad_mask, const int* level_lens,
                   int nlev, cudaStream_t stream) {
  if (T <= 0 || H <= 0 || Hkv <= 0 || H % Hkv != 0 || nlev < 0 || nlev > kMaxLevels || prefix < 0 || prefix > 64)
    return ncm_fail(NCM_EINVAL, "attention: bad arguments");
  AttnArgs a{};
  a.out = out;
  a.err = ctx->d_err;
  a.T = T;
  a.H = H;
  a.Hkv = Hkv;
  a.mode = mode;
  a.prefix = mode == 0 ? 0 : prefix;
  a.pad_mask = pad_mask;
  a.scale = 1.0f / std::sqrt(static_cast<float>(AT_D));
  if (mode != 0) {
    if (nlev <= 0) return ncm_fail(NCM_EINVAL, "attention: block masks need at least one level");
    a.nlev = nlev;
    int pos = prefix;
    for (int i = 0; i < nlev; ++i) {
      if (level_lens[i] <= 0) return ncm_fail(NCM_EINVAL, "attention: empty level");
      a.level_start[i] = pos;
      pos += level_lens[i];
    }
    a.level_start[nlev] = pos;
    if (pos != T) return ncm_fail(NCM_EINVAL, "attention: prefix + levels (%d) != T (%d)", pos, T);
  } else {
    a.nlev = 1;
    a.level_start[0] = 0;
    a.level_start[1] = T;
  }
  CUtensorMap tq, tk, tv;
  auto fn_ok = make_tmap_bf16_2d_strided(&tq, qkv, T, static_cast<uint64_t>(H) * AT_D, qkv_stride, AT_Q) &&
               make_tmap_bf16_2d_strided(&tk, qkv + static_cast<size_t>(H) * AT_D, T,
                                         static_cast<uint64_t>(Hkv) * AT_D, qkv_stride, AT_K) &&
               make_tmap_bf16_2d(&tv, vt, static_cast<uint64_t>(Hkv) * AT_D, T, 64);
  if (!fn_ok) return ncm_fail(NCM_EINVAL, "attention: tensor map encoding failed (T=%d, stride %lld)", T,
                              (long long)qkv_stride);
  static unsigned long long attr_set = 0;
  int dev = 0;
  NCM_CUDA_TRY(cudaGetDevice(&dev));
  if (dev >= 64 || !(attr_set & (1ull << dev))) {
    NCM_CUDA_TRY(cudaFuncSetAttribute(attention_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(ATTN_SMEM)));
    if (dev < 64) attr_set |= 1ull << dev;
  }
  dim3 grid((T + AT_Q - 1) / AT_Q, H);
  attention_bf16_kernel<<<grid, AT_THREADS, ATTN_SMEM, stream>>>(tq, tk, tv, a);
  NCM_CUDA_TRY(cudaGetLastError());
  return NCM_OK;
}

}  // namespace ncm
