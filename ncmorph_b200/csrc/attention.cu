// Fused masked GQA attention on tcgen05 (L3), for the NCM decoder forward.
//
// One CTA per (256 queries = two 128-query tiles Q0 and Q1, query head), both
// tiles sharing every K/V stage. Per key tile of 128:
//   S_i = Q_i . K^T       tcgen05.mma M=128 N=128 K=64, f32 in TMEM
//   softmax               one thread per query row (warps 2-5: Q0, 6-9: Q1),
//                         reading its whole S row from TMEM; P (bf16) into a
//                         128-byte-swizzled smem tile, the A operand of P.V
//   O_i += P_i . V        tcgen05.mma M=128 N=64 K=128, accumulated in TMEM
// The MMA warp interleaves the two tiles (P.V and the next S of one run while
// the other group computes its softmax). Key tiles that the mask removes
// entirely are never loaded, and CTAs launch heaviest first (late query
// tiles see the most keys). K tiles come straight from the fused QKV rows by
// TMA; V is read transposed ([kv_head*64 + d][t]) so both MMAs take K-major
// operands.
//
// Softmax in the log2 domain with a lagging reference maximum: after a row's
// first tile, a tile runs in one pass against the running reference (p may
// exceed 1; f32 sums and bf16 P carry it exactly up to 2^64); only a row
// without a reference, or whose maximum jumped by more than 2^64, makes its
// warp redo the tile in two passes (maximum first) and rescale O_i in TMEM.
//
// Score rounding follows ncmorph's bf16 attention (packages/kernels/root.zig:
// 546-548): the raw score q.k is rounded to bf16 before scaling. Probabilities
// enter P.V as bf16 and the context is rounded once to bf16 — within the bf16
// bar of the reference's materialised softmax, not bit-equal to it.
#include <cfloat>
#include <cmath>

#include "internal.h"
#include "ptx.cuh"

namespace ncm {
namespace {

constexpr int AT_Q = 128;       // queries per tile (two tiles per CTA)
constexpr int AT_K = 128;       // keys per tile
constexpr int AT_D = 64;        // head dim (fixed)
constexpr int AT_THREADS = 320;  // w0 TMA, w1 MMA, w2-5 softmax of Q0, w6-9 softmax of Q1
constexpr uint32_t AT_TMEM_COLS = 512;  // S_0, S_1: 128 cols each; O_0, O_1: 64 cols each
constexpr int kMaxLevels = 32;

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

constexpr int A2_STAGES = 3;
constexpr float kRescaleLog2 = 8.0f;

struct __align__(1024) Attn2Smem {
  uint8_t q[2][AT_Q * AT_D * 2];              // 2 x 16 KB
  uint8_t k[A2_STAGES][AT_K * AT_D * 2];      // 16 KB each
  uint8_t vt[A2_STAGES][2][AT_D * 64 * 2];    // 2 x 8 KB each: [64 d rows x 64 keys] per key half
  uint8_t p[2][2][AT_Q * 64 * 2];             // [query tile][key half] 16 KB, 128-byte swizzle
  uint64_t q_full;
  uint64_t kv_full[A2_STAGES];
  uint64_t kv_empty[A2_STAGES];
  uint64_t s_full[2];   // S_i computed
  uint64_t p_full[2];   // P_i written (and O_i rescaled): the 4 warps of group i
  uint64_t p_empty[2];  // P_i . V done: P_i and O_i free again
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};
constexpr size_t ATTN2_SMEM = sizeof(Attn2Smem) + 1024;
static_assert(ATTN2_SMEM <= 232448, "attention smem budget");

// One pass over a 128-key S row in tensor memory: p = 2^(bf16(s) * c_scale -
// m_use) for allowed keys (0 for masked ones) stored as bf16 into the row of
// the 128-byte-swizzled P tile (two 64-key halves), their sum added to rs.
// Returns the row's maximum bf16-rounded score times c_scale (log2 domain).
__device__ __forceinline__ float softmax_tile_pass(uint8_t (*p_half)[AT_Q * 64 * 2], uint32_t sbase, int row,
                                                   int k0, bool unmasked, int Pq, int lo, int hi,
                                                   unsigned long long pad_mask, float c_scale, float m_use,
                                                   float& rs) {
  const unsigned long long cs2 = f2_pack(c_scale, c_scale), nm2 = f2_pack(-m_use, -m_use);
  unsigned long long rs2 = f2_pack(0.f, 0.f);
  uint32_t mx2 = 0xFF80FF80u;  // bf16x2 -inf
#pragma unroll 1
  for (int c = 0; c < AT_K; c += 32) {
    uint32_t v[32];
    tmem_ld_x32(sbase + c, v);
    tmem_wait_ld();
    if (!unmasked) {
#pragma unroll
      for (int e = 0; e < 32; ++e)
        if (!key_allowed(k0 + c + e, Pq, lo, hi, pad_mask)) v[e] = __float_as_uint(-INFINITY);
    }
    uint8_t* prow = p_half[c >> 6] + row * 128;
    const int ch0 = (c & 63) >> 3;
#pragma unroll
    for (int q4 = 0; q4 < 4; ++q4) {  // four 16-byte chunks of 8 keys
      uint32_t w4[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int ii = q4 * 8 + e * 2;
        const uint32_t pr = cvt_bf16x2(__uint_as_float(v[ii]), __uint_as_float(v[ii + 1]));
        mx2 = bf16x2_max(mx2, pr);
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
  float r0, r1;
  f2_unpack(rs2, r0, r1);
  rs += r0 + r1;
  return fmaxf(bf16lo(mx2), bf16hi(mx2)) * c_scale;
}

struct TileSpan {
  int P, A, B;
  bool has;
  __device__ __forceinline__ bool need(int t) const { return has && tile_needed(t, P, A, B); }
};

__global__ void __launch_bounds__(AT_THREADS, 1)
    attention2_bf16_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                           const __grid_constant__ CUtensorMap tmVt, const AttnArgs args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  Attn2Smem& S = *reinterpret_cast<Attn2Smem*>(smem_raw + pad);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // CTAs are ordered heaviest first: causal masks give late query tiles the
  // most keys, so the last query-tile pair of every head launches first and
  // the light early tiles fill the tail of the grid
  const int n_qp = (args.T + 2 * AT_Q - 1) / (2 * AT_Q);
  const int qp = n_qp - 1 - static_cast<int>(blockIdx.x) / args.H;
  const int h = static_cast<int>(blockIdx.x) % args.H;
  const int q0 = qp * 2 * AT_Q;
  const int kvh = h / (args.H / args.Hkv);
  TileSpan span[2];
  int n_tiles_all = 0;
  for (int i = 0; i < 2; ++i) {
    span[i].has = q0 + i * AT_Q < args.T;
    cta_key_span(args, q0 + i * AT_Q, span[i].P, span[i].A, span[i].B);
    if (span[i].has) n_tiles_all = max(n_tiles_all, (max(span[i].B, span[i].P) + AT_K - 1) / AT_K);
  }
  auto need_any = [&](int t) { return span[0].need(t) || span[1].need(t); };

  if (threadIdx.x == 0) {
    mbar_init(&S.q_full, 1);
    for (int s = 0; s < A2_STAGES; ++s) {
      mbar_init(&S.kv_full[s], 1);
      mbar_init(&S.kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&S.s_full[i], 1);
      mbar_init(&S.p_full[i], 4);
      mbar_init(&S.p_empty[i], 1);
    }
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
  const uint32_t tmem = S.tmem_base;  // S_i at columns 128 i, O_i at 256 + 64 i
  volatile int* abort_flag = &S.abort_flag;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------ TMA producer
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmVt);
      mbar_arrive_expect_tx(&S.q_full, (span[1].has ? 2 : 1) * AT_Q * AT_D * 2);
      tma_load_2d(&tmQ, &S.q_full, S.q[0], h * AT_D, q0);
      if (span[1].has) tma_load_2d(&tmQ, &S.q_full, S.q[1], h * AT_D, q0 + AT_Q);
      int stage = 0;
      uint32_t phase = 0;
      bool issued[A2_STAGES];
      uint32_t iss_par[A2_STAGES];
      for (int s = 0; s < A2_STAGES; ++s) issued[s] = false, iss_par[s] = 0;
      bool ok = true;
      for (int t = 0; t < n_tiles_all && ok; ++t) {
        if (!need_any(t)) continue;
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
        if (++stage == A2_STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) {
        raise_abort_attn(abort_flag, args.err);
        mbar_wait(&S.q_full, 0, nullptr);
        for (int s = 0; s < A2_STAGES; ++s)
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
      auto next_needed = [&](int t) {
        for (int u = t + 1; u < n_tiles_all; ++u)
          if (need_any(u)) return u;
        return -1;
      };
      auto issue_s = [&](int i, int st) {
        const uint32_t qa = smem_u32(S.q[i]), ka = smem_u32(S.k[st]);
#pragma unroll
        for (int k = 0; k < AT_D / 16; ++k)
          tc_mma_f16(tmem + i * AT_K, smem_desc_k_sw128(qa + k * 32), smem_desc_k_sw128(ka + k * 32), idesc_s,
                     k != 0 ? 1u : 0u);
        tc_commit(&S.s_full[i]);
      };
      int cur = next_needed(-1);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t npv[2] = {0u, 0u};  // P.V products issued per query tile
      if (ok && cur >= 0) {
        if (!mbar_wait(&S.kv_full[0], 0, abort_flag)) ok = false;
        tc_fence_after();
        for (int i = 0; ok && i < 2; ++i)
          if (span[i].need(cur)) issue_s(i, 0);
      }
      while (ok && cur >= 0) {
        const int nxt = next_needed(cur);
        int nstage = stage + 1;
        uint32_t nphase = phase;
        if (nstage == A2_STAGES) nstage = 0, nphase ^= 1u;
        bool kv_ready = false;
        for (int i = 0; i < 2; ++i) {
          if (span[i].need(cur)) {
            // O_i (+)= P_i . V_cur once the softmax of group i released the tile
            if (!mbar_wait(&S.p_full[i], npv[i] & 1u, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < AT_K / 16; ++kk) {
              const uint32_t pa = smem_u32(S.p[i][kk >> 2]) + (kk & 3) * 32;
              const uint32_t va = smem_u32(S.vt[stage][kk >> 2]) + (kk & 3) * 32;
              tc_mma_f16(tmem + 2 * AT_K + i * AT_D, smem_desc_k_sw128(pa), smem_desc_k_sw128(va), idesc_o,
                         (npv[i] > 0 || kk != 0) ? 1u : 0u);
            }
            tc_commit(&S.p_empty[i]);
            ++npv[i];
          }
          if (nxt >= 0 && span[i].need(nxt)) {
            // the S_i buffer is free: its softmax finished reading (p_full waited above, or long ago)
            if (!kv_ready) {
              if (!mbar_wait(&S.kv_full[nstage], nphase, abort_flag)) {
                ok = false;
                break;
              }
              tc_fence_after();
              kv_ready = true;
            }
            issue_s(i, nstage);
          }
        }
        if (!ok) break;
        tc_commit(&S.kv_empty[stage]);
        cur = nxt;
        stage = nstage;
        phase = nphase;
      }
      if (!ok) {
        raise_abort_attn(abort_flag, args.err);
        tc_commit(&S.drain);
        mbar_wait(&S.drain, 0, nullptr);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int gi = (warp - 2) >> 2;  // query tile of this warp group
    const int qw = warp & 3;
    const int row = qw * 32 + lane;
    const int q = q0 + gi * AT_Q + row;
    const TileSpan sp = span[gi];
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
    const uint32_t lane_base = static_cast<uint32_t>(qw * 32) << 16;
    const uint32_t sbase = tmem + lane_base + gi * AT_K;
    const uint32_t obase = tmem + lane_base + 2 * AT_K + gi * AT_D;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    uint32_t j = 0;
    for (int t = 0; t < n_tiles_all; ++t) {
      if (!sp.need(t)) continue;
      // every outcome that guards a warp-wide (.sync.aligned) TMEM access is made
      // uniform across the warp, so no lane can take a branch its neighbours skip
      if (!__all_sync(0xffffffffu, mbar_wait(&S.s_full[gi], j & 1u, abort_flag))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int k0 = t * AT_K;
      const bool unmasked = __all_sync(0xffffffffu, k0 >= Pq && k0 >= lo && k0 + AT_K <= hi);
      // P_i and O_i are free once P.V of this group's previous tile completed
      if (j > 0 && !__all_sync(0xffffffffu, mbar_wait(&S.p_empty[gi], (j - 1) & 1u, abort_flag))) {
        ok = false;
        break;
      }
      // One pass against the running reference m_used when every row of the
      // warp has one: probabilities may then exceed 1 (the reference lags the
      // true maximum), which f32 sums and bf16 P carry exactly up to 2^64. A
      // row without a reference yet, or whose maximum jumped past m_used + 64,
      // makes the warp redo the tile in two passes with a rescale.
      bool two_pass = __any_sync(0xffffffffu, m_used == -INFINITY);
      if (!two_pass) {
        float rs = 0.f;
        const float mt = softmax_tile_pass(S.p[gi], sbase, row, k0, unmasked, Pq, lo, hi, args.pad_mask, c_scale,
                                           m_used, rs);
        if (__any_sync(0xffffffffu, mt > m_used + 64.f)) {
          two_pass = true;
        } else {
          l += rs;
        }
      }
      if (two_pass) {
        // pass 1: row maximum of the raw scores (rounding to bf16 is monotonic)
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll 1
        for (int c = 0; c < AT_K; c += 32) {
          uint32_t v[32];
          tmem_ld_x32(sbase + c, v);
          tmem_wait_ld();
          if (!unmasked) {
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (!key_allowed(k0 + c + e, Pq, lo, hi, args.pad_mask)) v[e] = __float_as_uint(-INFINITY);
          }
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            mx0 = fmaxf(mx0, __uint_as_float(v[e]));
            mx1 = fmaxf(mx1, __uint_as_float(v[e + 1]));
          }
        }
        const float mt = bf16lo(cvt_bf16x2(fmaxf(mx0, mx1), 0.f)) * c_scale;
        const bool rescale = mt > m_used + kRescaleLog2;  // m_used = -inf: any finite maximum
        const float m_new = rescale ? mt : m_used;
        const float m_use = m_new == -INFINITY ? 0.f : m_new;
        const float alpha = rescale ? ex2_approx(m_used - m_new) : 1.f;  // -inf -> 0
        // pass 2: t = bf16(s) * scale * log2(e) - m, p = 2^t (<= 256), bf16 into P_i
        float rs = 0.f;
        softmax_tile_pass(S.p[gi], sbase, row, k0, unmasked, Pq, lo, hi, args.pad_mask, c_scale, m_use, rs);
        if (j > 0 && __any_sync(0xffffffffu, rescale)) {
          // O_i row *= alpha in tensor memory before the next P.V accumulates into
          // it (the whole warp executes the TMEM accesses; rows without a rescale
          // have alpha = 1)
#pragma unroll 1
          for (int c = 0; c < AT_D; c += 32) {
            uint32_t v[32];
            tmem_ld_x32(obase + c, v);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * alpha);
            tmem_st_x32(obase + c, v);
          }
          tmem_wait_st();
        }
        l = l * alpha + rs;
        m_used = m_new;
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.p_full[gi]);
      ++j;
    }
    if (ok && j > 0) ok = __all_sync(0xffffffffu, mbar_wait(&S.p_empty[gi], (j - 1) & 1u, abort_flag));
    if (!ok) raise_abort_attn(abort_flag, args.err);
    uint16_t* dst = args.out + static_cast<size_t>(q) * args.H * AT_D + h * AT_D;
    if (ok && j > 0) {
      // the whole warp reads its O rows; rows past T only skip the stores
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll 1
      for (int c = 0; c < AT_D; c += 32) {
        uint32_t v[32];
        tmem_ld_x32(obase + c, v);
        tmem_wait_ld();
        if (q < args.T) {
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            uint4 w;
            w.x = cvt_bf16x2(__uint_as_float(v[e + 0]) * inv, __uint_as_float(v[e + 1]) * inv);
            w.y = cvt_bf16x2(__uint_as_float(v[e + 2]) * inv, __uint_as_float(v[e + 3]) * inv);
            w.z = cvt_bf16x2(__uint_as_float(v[e + 4]) * inv, __uint_as_float(v[e + 5]) * inv);
            w.w = cvt_bf16x2(__uint_as_float(v[e + 6]) * inv, __uint_as_float(v[e + 7]) * inv);
            *reinterpret_cast<uint4*>(dst + c + e) = w;
          }
        }
      }
    } else if (ok && q < args.T) {
      // no allowed key at all (a fully masked row): the context is zero
#pragma unroll
      for (int c = 0; c < AT_D; c += 8) *reinterpret_cast<uint4*>(dst + c) = make_uint4(0u, 0u, 0u, 0u);
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
    NCM_CUDA_TRY(cudaFuncSetAttribute(attention2_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(ATTN2_SMEM)));
    if (dev < 64) attr_set |= 1ull << dev;
  }
  const int n_qp = (T + 2 * AT_Q - 1) / (2 * AT_Q);
  attention2_bf16_kernel<<<n_qp * H, AT_THREADS, ATTN2_SMEM, stream>>>(tq, tk, tv, a);
  NCM_CUDA_TRY(cudaGetLastError());
  return NCM_OK;
}

}  // namespace ncm
