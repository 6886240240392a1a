// Fused masked GQA attention on tcgen05 (L3), for the NCM decoder forward.
//
// One CTA per (256 queries = two 128-query tiles Q0 and Q1, query head), both
// tiles sharing every K/V stage. Per key tile of 128:
//   S_i = Q_i . K^T       tcgen05.mma M=128 N=128 K=64, f32 in TMEM
//   softmax               one thread per query row (warps 2-5: Q0, 6-9: Q1),
//                         reading its whole S row from TMEM; P (bf16) into a
//                         128-byte-swizzled smem tile, the A operand of P.V
//   O_i += P_i . V        tcgen05.mma M=128 N=64 K=128, accumulated in TMEM
// A group's S buffer is released (s_free) as soon as its softmax threads hold
// the scores in registers, so the MMA warp issues the next tile's S for both
// groups while their exponentials run, then each group's P.V when its P is
// written (p_full); a softmax pass therefore rarely waits for its S. Key tiles
// that the mask removes entirely are never loaded, and CTAs launch heaviest
// first (late query tiles see the most keys). K tiles come straight from the fused QKV rows by
// TMA; V is read transposed ([kv_head*64 + d][t]) so both MMAs take K-major
// operands.
//
// Softmax in the log2 domain with a lagging reference maximum: each softmax
// thread reads its whole S row into registers (one wait), takes the row
// maximum there, and computes p against the running reference m, which moves
// only when the row maximum exceeds it by more than 2^64 (p may exceed 1;
// f32 sums and bf16 P carry it exactly); a moved reference rescales the row
// of O_i in TMEM.
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
  int window;      // causal mode: keys q - window < k <= q (0: no window)
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

// Key intervals the CTA's queries may see: [0, P) and [A, B). A sliding
// window moves A up to the first query's earliest key.
__device__ __forceinline__ void cta_key_span(const AttnArgs& a, int q0, int& P, int& A, int& B) {
  const int qmax = min(q0 + AT_Q - 1, a.T - 1);
  if (a.mode == 0) {
    P = 0;
    A = a.window > 0 ? max(q0 - a.window + 1, 0) : 0;
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

__device__ __forceinline__ void raise_abort_attn(volatile int* abort_flag, int* err) {
  *abort_flag = 1;
  atomicOr(err, kErrWaitTimeout);
}

constexpr int A2_STAGES = 3;
constexpr float kLagLog2 = 64.0f;  // largest lag of the reference maximum (log2 domain)

struct __align__(1024) Attn2Smem {
  uint8_t q[2][AT_Q * AT_D * 2];              // 2 x 16 KB
  uint8_t k[A2_STAGES][AT_K * AT_D * 2];      // 16 KB each
  uint8_t vt[A2_STAGES][2][AT_D * 64 * 2];    // 2 x 8 KB each: [64 d rows x 64 keys] per key half
  uint8_t p[2][2][AT_Q * 64 * 2];             // [query tile][key half] 16 KB, 128-byte swizzle
  uint64_t q_full;
  uint64_t kv_full[A2_STAGES];
  uint64_t kv_empty[A2_STAGES];
  uint64_t s_full[2];   // S_i computed
  uint64_t s_free[2];   // S_i read into registers: the 4 warps of group i (the next S_i may overwrite it)
  uint64_t p_full[2];   // P_i written (and O_i rescaled): the 4 warps of group i
  uint64_t p_empty[2];  // P_i . V done: P_i and O_i free again
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};
constexpr size_t ATTN2_SMEM = sizeof(Attn2Smem) + 1024;
static_assert(ATTN2_SMEM <= 232448, "attention smem budget");

// The row's 128 scores from tensor memory (four loads, one wait), rounded to
// bf16 pairs (ncmorph rounds the raw score q.k to bf16), masked keys set to
// bf16 -inf, and the row maximum of the rounded scores times c_scale (log2
// domain). Four independent maximum chains keep the dependency depth short.
// A masked tile's allowed keys are the row's window [lo, hi) plus, in tile 0,
// the unpadded prefix keys [0, Pq) (Pq <= 64).
__device__ __forceinline__ float load_scores(uint32_t sbase, int k0, bool unmasked, int Pq, int lo, int hi,
                                             unsigned long long pad_mask, float c_scale,
                                             uint32_t (&pr)[AT_K / 2]) {
  {
    uint32_t v[AT_K];
#pragma unroll
    for (int c = 0; c < AT_K; c += 32) tmem_ld_x32(sbase + c, *reinterpret_cast<uint32_t(*)[32]>(&v[c]));
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < AT_K / 2; ++i) pr[i] = cvt_bf16x2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
  }
  if (!unmasked) {
    const int a = lo - k0, b = hi - k0;
    uint32_t m[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const int l0 = max(a - 32 * w, 0), h0 = min(b - 32 * w, 32);
      m[w] = h0 > l0 ? (h0 >= 32 ? 0xFFFFFFFFu : (1u << h0) - 1u) & ~((1u << l0) - 1u) : 0u;
    }
    if (k0 < Pq) {
      const unsigned long long pm = ~pad_mask & (Pq >= 64 ? ~0ull : (1ull << Pq) - 1ull);
      m[0] |= static_cast<uint32_t>(pm);
      m[1] |= static_cast<uint32_t>(pm >> 32);
    }
#pragma unroll
    for (int i = 0; i < AT_K / 2; ++i) {
      const uint32_t b2 = (m[i >> 4] >> ((2 * i) & 31)) & 3u;
      const uint32_t keep = ((b2 & 1u) ? 0x0000FFFFu : 0u) | ((b2 & 2u) ? 0xFFFF0000u : 0u);
      pr[i] = (pr[i] & keep) | (0xFF80FF80u & ~keep);
    }
  }
  uint32_t mx[4] = {0xFF80FF80u, 0xFF80FF80u, 0xFF80FF80u, 0xFF80FF80u};  // bf16x2 -inf
#pragma unroll
  for (int i = 0; i < AT_K / 2; ++i) mx[i & 3] = bf16x2_max(mx[i & 3], pr[i]);
  const uint32_t m2 = bf16x2_max(bf16x2_max(mx[0], mx[1]), bf16x2_max(mx[2], mx[3]));
  return fmaxf(bf16lo(m2), bf16hi(m2)) * c_scale;
}

// p = 2^(bf16(s) * c_scale - m_use) for the row's 128 keys (masked keys give
// 2^-inf = 0), stored as bf16 into the row of the 128-byte-swizzled P tile
// (two 64-key halves); returns the f32 sum of the p (four partial sums).
__device__ __forceinline__ float exp_pass(uint8_t (*p_half)[AT_Q * 64 * 2], int row, const uint32_t (&pr)[AT_K / 2],
                                          float c_scale, float m_use) {
  const unsigned long long cs2 = f2_pack(c_scale, c_scale), nm2 = f2_pack(-m_use, -m_use);
  unsigned long long rs2[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) rs2[e] = f2_pack(0.f, 0.f);
#pragma unroll
  for (int c8 = 0; c8 < AT_K / 8; ++c8) {  // sixteen 16-byte chunks of 8 keys
    uint32_t w4[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint32_t p2 = pr[c8 * 4 + e];
      const unsigned long long t2 = f2_fma(f2_pack(bf16lo(p2), bf16hi(p2)), cs2, nm2);
      float t0, t1;
      f2_unpack(t2, t0, t1);
      const float p0 = ex2_approx(t0), p1 = ex2_approx(t1);
      w4[e] = cvt_bf16x2(p0, p1);
      rs2[e] = f2_add(rs2[e], f2_pack(p0, p1));
    }
    const int sw = (c8 & 7) ^ (row & 7);  // 128-byte swizzle: 16-byte chunk XOR row%8
    *reinterpret_cast<uint4*>(p_half[c8 >> 3] + row * 128 + sw * 16) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
  }
  float r0, r1;
  f2_unpack(f2_add(f2_add(rs2[0], rs2[1]), f2_add(rs2[2], rs2[3])), r0, r1);
  return r0 + r1;
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
      mbar_init(&S.s_free[i], 4);
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
  // the prologue above overlaps the previous kernel's tail (programmatic launch)
  pdl_wait();
  pdl_launch_dependents();
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
      // Shared-memory descriptors are computed once: a tile's descriptor is its
      // base's plus the tile offset / 16, and a 16-element K step adds 32 B
      // (2 in the address field), so each MMA costs one 64-bit add per operand.
      const uint64_t dq0 = smem_desc_k_sw128(smem_u32(S.q[0]));
      const uint64_t dk0 = smem_desc_k_sw128(smem_u32(S.k[0]));
      const uint64_t dv0 = smem_desc_k_sw128(smem_u32(S.vt[0][0]));
      const uint64_t dp0 = smem_desc_k_sw128(smem_u32(S.p[0][0]));
      constexpr uint64_t kQ16 = AT_Q * AT_D * 2 / 16, kK16 = AT_K * AT_D * 2 / 16;
      constexpr uint64_t kH16 = AT_D * 64 * 2 / 16, kP16 = AT_Q * 64 * 2 / 16;  // V^T and P half tiles
      auto issue_s = [&](int i, int st) {
        const uint64_t da = dq0 + i * kQ16, db = dk0 + st * kK16;
        const uint32_t d = tmem + i * AT_K;
#pragma unroll
        for (int k = 0; k < AT_D / 16; ++k) tc_mma_f16(d, da + 2 * k, db + 2 * k, idesc_s, k != 0 ? 1u : 0u);
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
        // S of the next tile first: a group's S buffer is free as soon as its
        // softmax holds the current scores in registers (s_free), so the next
        // S is computed while that softmax still runs its exponentials. (A
        // group without the current tile last read its S before a p_full that
        // was already waited for.)
        if (nxt >= 0) {
          if (!mbar_wait(&S.kv_full[nstage], nphase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          for (int i = 0; i < 2; ++i) {
            if (!span[i].need(nxt)) continue;
            if (span[i].need(cur) && !mbar_wait(&S.s_free[i], npv[i] & 1u, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_s(i, nstage);
          }
          if (!ok) break;
        }
        for (int i = 0; i < 2; ++i) {
          if (!span[i].need(cur)) continue;
          // O_i (+)= P_i . V_cur once the softmax of group i wrote P_i
          if (!mbar_wait(&S.p_full[i], npv[i] & 1u, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = dp0 + 2 * i * kP16, db = dv0 + 2 * stage * kH16;
          const uint32_t d = tmem + 2 * AT_K + i * AT_D;
          const uint32_t acc0 = npv[i] > 0 ? 1u : 0u;
#pragma unroll
          for (int kk = 0; kk < AT_K / 16; ++kk)
            tc_mma_f16(d, da + (kk >> 2) * kP16 + 2 * (kk & 3), db + (kk >> 2) * kH16 + 2 * (kk & 3), idesc_o,
                       kk != 0 ? 1u : acc0);
          tc_commit(&S.p_empty[i]);
          ++npv[i];
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
      lo = args.window > 0 ? max(q - args.window + 1, 0) : 0;
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
      // The row maximum is known before any exponential (the scores stay in
      // registers), so every tile takes one pass. The reference m_used lags
      // the true maximum: it moves (and O_i is rescaled) only when a tile's
      // maximum exceeds it by more than 2^kLagLog2, so p may exceed 1, which
      // f32 sums and bf16 P carry exactly.
      uint32_t pr[AT_K / 2];
      const float mt = load_scores(sbase, k0, unmasked, Pq, lo, hi, args.pad_mask, c_scale, pr);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.s_free[gi]);  // S_i may now be overwritten by the next tile's S
      // P_i and O_i are free once P.V of this group's previous tile completed
      if (j > 0 && !__all_sync(0xffffffffu, mbar_wait(&S.p_empty[gi], (j - 1) & 1u, abort_flag))) {
        ok = false;
        break;
      }
      const bool rescale = mt > m_used + kLagLog2;  // m_used = -inf: any finite maximum
      const float m_new = rescale ? mt : m_used;
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = rescale ? ex2_approx(m_used - m_new) : 1.f;  // -inf -> 0
      const float rs = exp_pass(S.p[gi], row, pr, c_scale, m_use);
      if (j > 0 && __any_sync(0xffffffffu, rescale)) {
        // O_i row *= alpha in tensor memory before the next P.V accumulates into
        // it (the whole warp executes the TMEM accesses; rows without a rescale
        // have alpha = 1)
        uint32_t v[AT_D];
        tmem_ld_x32(obase, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
        tmem_ld_x32(obase + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < AT_D; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * alpha);
        tmem_st_x32(obase, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
        tmem_st_x32(obase + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
        tmem_wait_st();
      }
      l = l * alpha + rs;
      m_used = m_new;
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
                   int nlev, int window, cudaStream_t stream) {
  if (T <= 0 || H <= 0 || Hkv <= 0 || H % Hkv != 0 || nlev < 0 || nlev > kMaxLevels ||
      (mode != 0 && (prefix < 0 || prefix > 64)) || window < 0 || (window > 0 && mode != 0))
    return ncm_fail(NCM_EINVAL, "attention: bad arguments");
  AttnArgs a{};
  a.out = out;
  a.err = ctx->d_err;
  a.T = T;
  a.H = H;
  a.Hkv = Hkv;
  a.mode = mode;
  a.window = window;
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
  static DeviceFlags attr_set;
  int dev = 0;
  NCM_CUDA_TRY(cudaGetDevice(&dev));
  if (!attr_set.test(dev)) {
    NCM_CUDA_TRY(cudaFuncSetAttribute(attention2_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(ATTN2_SMEM)));
    attr_set.set(dev);
  }
  const int n_qp = (T + 2 * AT_Q - 1) / (2 * AT_Q);
  NCM_CUDA_TRY(launch_pdl(attention2_bf16_kernel, dim3(n_qp * H), dim3(AT_THREADS), ATTN2_SMEM, stream, 1, tq, tk, tv,
                          a));
  return NCM_OK;
}

}  // namespace ncm
