// bf16 linear layer y = x . W^T (+ bias) on tcgen05 tensor cores (L1).
//
// Same pipeline skeleton as the RVQ distance kernel: persistent CTAs (one per
// SM), warp 0 issues TMA loads of 128-byte-swizzled K-major tiles into a
// multi-stage mbarrier ring, warp 1 issues tcgen05.mma (bf16 x bf16 -> f32 in
// tensor memory), warps 2-9 drain the double-buffered TMEM accumulator (two
// warps per TMEM lane quarter, alternating 16-column chunks, so twice the
// global accesses are in flight), add the bias in f32, round once to bf16 and
// store.
//
// Skinny problems (M <= 64 tokens: decode-time GEMV shapes) run "swapped":
// the 128-row MMA operand is the weight and the token rows form the narrow N
// side of the instruction (16/32/64), so the kernel streams W once at HBM
// speed instead of padding the tokens to 128 rows.
#include <algorithm>

#include "internal.h"
#include "ptx.cuh"

namespace ncm {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int EPI_WARPS = 8;  // two per TMEM lane quarter, interleaving 16-column chunks
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr int A_BYTES = BM * BK * 2;

// PAIR: clusters of two CTAs share each MMA (tcgen05 cta_group::2, M = 256):
// each CTA loads its own 128 rows of A and half of the BN-row B tile, the even
// CTA issues the MMAs, and each CTA's TMEM receives its own 128 rows.
template <int BN, bool PAIR = false>
struct GemmCfg {
  static constexpr int B_ROWS = PAIR ? BN / 2 : BN;
  static constexpr int B_BYTES = B_ROWS * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (196608 / STAGE_BYTES) > 8 ? 8 : (196608 / STAGE_BYTES);
  static constexpr uint32_t STAGE_TX = PAIR ? 2u * STAGE_BYTES : STAGE_BYTES;  // counted on the leader
  static constexpr uint32_t TMEM_COLS = (2 * BN) < 32 ? 32 : 2 * BN;
};

template <int BN, bool PAIR = false>
struct __align__(1024) GemmSmem {
  uint8_t a[GemmCfg<BN, PAIR>::STAGES][A_BYTES];
  uint8_t b[GemmCfg<BN, PAIR>::STAGES][GemmCfg<BN, PAIR>::B_BYTES];
  uint64_t full[GemmCfg<BN, PAIR>::STAGES];
  uint64_t empty[GemmCfg<BN, PAIR>::STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};

struct LinearArgs {
  const uint16_t* bias;  // [N] or null
  uint16_t* y;           // [M,N] bf16 (or null)
  float* y_f32;          // [M,N] f32 (or null)
  int* err;
  int M, N, K;
  int tiles_a, tiles_b;  // tiles along the 128-row operand and the BN operand
  // split-K (swapped form only): unit = (tile, split); split s sums k-chunks
  // [s * nk_split, (s + 1) * nk_split) into f32 partials part[s][m][n]
  int ksplit, nk_split;
  float* part;
  int a_fast;            // raster: 1 = consecutive tiles walk the A-operand tiles
  int vec_ok;            // y rows are 16-byte aligned (N % 8 == 0)
  int mode;              // 0 plain, 1 SwiGLU (y[M,F]), 2 residual add into y, 3 kernel-3 convolution
  int F;                 // SwiGLU width (mode 1): gate rows [0,F), up rows [F,2F) of W
  // mode 3: K = 3 * nk_tap * BK; K-chunk kc reads tap kc / nk_tap, i.e. the
  // A rows shifted by tap - 1 (the padded copy supplies the zeros)
  int taps, nk_tap;
  ConvEpilogue conv;
  SegMap map;
  // mode 4 (codebook-tied head logits into y_f32): logits = fmaf(2 s, acc, -c[n])
  // with per-code offsets c [N] = s E_sq - bias and scal[2] = -2 s on the device
  // (s = exp(log_inv_T) / d_scale)
  const float* head_c;
  const float* head_scal;
  // mode 5 (fused QKV projection): RoPE on the Q and K columns (n < voff) with
  // per-token tables cos/sin [M, 64]; V columns also written transposed to
  // vt [(n - voff), M]
  const uint16_t* rope_cos;  // bf16(cos), bf16(sin) tables [M, 64]
  const uint16_t* rope_sin;
  uint16_t* vt;
  int voff;
};

__device__ __forceinline__ void tile_coords(int tile, const LinearArgs& a, int& ta, int& tb) {
  if (a.a_fast) {
    tb = tile / a.tiles_a;
    ta = tile - tb * a.tiles_a;
  } else {
    ta = tile / a.tiles_b;
    tb = tile - ta * a.tiles_b;
  }
}

template <int BN, bool SWAP, bool PAIR>
__global__ void __launch_bounds__(THREADS, 1)
    linear_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                       const LinearArgs args) {
  static_assert(!(SWAP && PAIR), "the swapped (skinny) form runs on single CTAs");
  using Cfg = GemmCfg<BN, PAIR>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  GemmSmem<BN, PAIR>& S = *reinterpret_cast<GemmSmem<BN, PAIR>*>(smem_raw + pad);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nk = (args.K + BK - 1) / BK;
  const int n_tiles = args.tiles_a * args.tiles_b;
  const int ksplit = SWAP ? args.ksplit : 1;
  const int n_units = n_tiles * ksplit;  // unit u: tile u / ksplit, k split u % ksplit
  auto k_range = [&](int unit, int& k0, int& k1) {
    if (ksplit == 1) {
      k0 = 0;
      k1 = nk;
      return;
    }
    const int sp = unit % ksplit;
    k0 = sp * args.nk_split;
    k1 = min(nk, k0 + args.nk_split);
  };
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;  // 0 = leader (issues the pair's MMAs)
  const int cid = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int ncl = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  // first row of the 128-row A block this CTA owns in tile-row ta
  auto a_row0 = [&](int ta) { return PAIR ? ta * 2 * BM + static_cast<int>(rank) * BM : ta * BM; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&S.tfull[b], 1);
      mbar_init(&S.tempty[b], PAIR ? 2 * EPI_WARPS : EPI_WARPS);  // a pair's leader hears both epilogues
    }
    mbar_init(&S.drain, 1);
    S.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(&S.tmem_base, Cfg::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(&S.tmem_base, Cfg::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  // a pair's barriers must be initialised in both CTAs before either signals the other
  if constexpr (PAIR) cluster_sync_all();
  tc_fence_after();
  // the prologue above overlaps the previous kernel's tail (programmatic launch)
  pdl_wait();
  pdl_launch_dependents();
  const uint32_t tmem = S.tmem_base;
  volatile int* abort_flag = &S.abort_flag;
  auto abort_all = [&]() {
    *abort_flag = 1;
    atomicOr(args.err, kErrWaitTimeout);
    if constexpr (PAIR) st_shared_cluster_u32(mapa_shared(smem_u32(&S.abort_flag), rank ^ 1u), 1u);
  };

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      bool issued[STAGES];
      uint32_t issued_parity[STAGES];
      for (int s = 0; s < STAGES; ++s) issued[s] = false, issued_parity[s] = 0;
      bool ok = true;
      for (int unit = cid; ok && unit < n_units; unit += ncl) {
        int ta, tb, k0, k1;
        tile_coords(unit / ksplit, args, ta, tb);
        k_range(unit, k0, k1);
        const int ar = a_row0(ta);
        for (int kc = k0; kc < k1; ++kc) {
          if (!mbar_wait(&S.empty[stage], phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          // A: this CTA's rows (conv: row -1 of the first tile is outside the
          // tensor and TMA fills it with zeros)
          int ax = kc * BK, ay = ar;
          if (args.taps > 1) {
            const int tap = kc / args.nk_tap;
            ax = (kc - tap * args.nk_tap) * BK;
            ay = ar + tap - 1;
          }
          if constexpr (PAIR) {
            // both CTAs' copies complete on the leader's full barrier, which
            // alone posts the expected bytes; B: this CTA's half of the tile
            // (SwiGLU: the leader the gate rows, the follower the up rows)
            if (rank == 0) mbar_arrive_expect_tx(&S.full[stage], Cfg::STAGE_TX);
            const uint32_t fb = mapa_shared(smem_u32(&S.full[stage]), 0);
            tma_load_2d_pair(&tmA, fb, S.a[stage], ax, ay);
            const int by = args.mode == 1 ? (rank == 0 ? 0 : args.F) + tb * (BN / 2)
                                          : tb * BN + static_cast<int>(rank) * (BN / 2);
            tma_load_2d_pair(&tmB, fb, S.b[stage], kc * BK, by);
          } else {
            mbar_arrive_expect_tx(&S.full[stage], Cfg::STAGE_TX);
            tma_load_2d(&tmA, &S.full[stage], S.a[stage], ax, ay);
            if (args.mode == 1) {
              // gate rows and the matching up rows side by side in one tile
              tma_load_2d(&tmB, &S.full[stage], S.b[stage], kc * BK, tb * (BN / 2));
              tma_load_2d(&tmB, &S.full[stage], S.b[stage] + (BN / 2) * BK * 2, kc * BK, args.F + tb * (BN / 2));
            } else {
              tma_load_2d(&tmB, &S.full[stage], S.b[stage], kc * BK, tb * BN);
            }
          }
          issued[stage] = true;
          issued_parity[stage] = phase;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        abort_all();
        // let this thread's copies land before the CTA exits (a pair's
        // follower cannot observe the leader's barrier: it waits 20 us)
        if (!PAIR || rank == 0) {
          for (int s = 0; s < STAGES; ++s)
            if (issued[s]) mbar_wait(&S.full[s], issued_parity[s], nullptr);
        } else {
          __nanosleep(20000);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && (!PAIR || rank == 0)) {
      const uint32_t idesc = idesc_bf16_f32(PAIR ? 2 * BM : BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t acc_it = 0;
      bool ok = true;
      for (int unit = cid; ok && unit < n_units; unit += ncl) {
        int k0, k1;
        k_range(unit, k0, k1);
        const uint32_t b = acc_it & 1u;
        const uint32_t ap = (acc_it >> 1) & 1u;
        if (!mbar_wait(&S.tempty[b], ap ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t dt = tmem + b * BN;
        for (int kc = k0; kc < k1; ++kc) {
          if (!mbar_wait(&S.full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(S.a[stage]);
          const uint32_t b0 = smem_u32(S.b[stage]);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            if constexpr (PAIR)
              tc_mma_f16_pair(dt, smem_desc_k_sw128(a0 + k * 32), smem_desc_k_sw128(b0 + k * 32), idesc,
                              (kc != k0 || k != 0) ? 1u : 0u);
            else
              tc_mma_f16(dt, smem_desc_k_sw128(a0 + k * 32), smem_desc_k_sw128(b0 + k * 32), idesc,
                         (kc != k0 || k != 0) ? 1u : 0u);
          }
          // the stage is free again (in both CTAs of a pair)
          if constexpr (PAIR)
            tc_commit_pair(&S.empty[stage], 0x3);
          else
            tc_commit(&S.empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if constexpr (PAIR)
          tc_commit_pair(&S.tfull[b], 0x3);
        else
          tc_commit(&S.tfull[b]);
        ++acc_it;
      }
      if (!ok) {
        abort_all();
        if constexpr (PAIR)
          tc_commit_pair(&S.drain, 0x1);
        else
          tc_commit(&S.drain);
        mbar_wait(&S.drain, 0, nullptr);
      }
    }
  } else {
    const int q = warp & 3;
    const int c0 = ((warp - 2) >> 2) * 16;  // first 16-column chunk of this warp; chunks step by 32
    uint32_t acc_it = 0;
    bool ok = true;
    for (int unit = cid; unit < n_units; unit += ncl) {
      int ta, tb;
      tile_coords(unit / ksplit, args, ta, tb);
      const uint32_t b = acc_it & 1u;
      const uint32_t ap = (acc_it >> 1) & 1u;
      if (!__all_sync(0xffffffffu, mbar_wait(&S.tfull[b], ap, abort_flag))) {  // warp-uniform: TMEM loads follow
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t tbase = tmem + (static_cast<uint32_t>(q * 32) << 16) + b * BN;
      const int arow = a_row0(ta) + q * 32 + lane;  // row of the 128-row operand this thread owns
      if (!SWAP && args.mode == 1) {
        // SwiGLU (decoder.zig:205-210): y = bf16(bf16(silu(bf16(g))) * bf16(u))
        const int m = arow;
        const int n0 = tb * (BN / 2);
#pragma unroll 1
        for (int c = c0; c < BN / 2; c += 32) {
          uint32_t g[16], u[16];
          tmem_ld_x16(tbase + c, g);
          tmem_ld_x16(tbase + BN / 2 + c, u);
          tmem_wait_ld();
          if (m < args.M) {
            uint32_t w8[8];
#pragma unroll
            for (int j = 0; j < 16; j += 2) {
              const uint32_t gp = cvt_bf16x2(__uint_as_float(g[j]), __uint_as_float(g[j + 1]));
              const uint32_t up = cvt_bf16x2(__uint_as_float(u[j]), __uint_as_float(u[j + 1]));
              const float g0 = bf16lo(gp), g1 = bf16hi(gp);
              // silu(g) = g / (1 + e^-g), e^-g = 2^(-g log2 e)
              const float s0 = __fdividef(g0, 1.0f + ex2_approx(-1.4426950408889634f * g0));
              const float s1 = __fdividef(g1, 1.0f + ex2_approx(-1.4426950408889634f * g1));
              const uint32_t sp = cvt_bf16x2(s0, s1);
              w8[j / 2] = cvt_bf16x2(bf16lo(sp) * bf16lo(up), bf16hi(sp) * bf16hi(up));
            }
            uint16_t* dst = args.y + static_cast<size_t>(m) * args.F + n0 + c;
            *reinterpret_cast<uint4*>(dst) = make_uint4(w8[0], w8[1], w8[2], w8[3]);
            *reinterpret_cast<uint4*>(dst + 8) = make_uint4(w8[4], w8[5], w8[6], w8[7]);
          }
        }
      } else if (!SWAP && args.mode == 5) {
        // QKV epilogue: y = bf16(acc + bias); per 64-column head, rotate_head in
        // bf16 mode (packages/kernels/root.zig:615-633) on the pair (d, d + 32)
        // for Q and K heads, and V heads also stored transposed for the
        // attention's P.V operand. This warp takes the pairs whose first
        // column is at c0 + 64 j (c0 = 0 or 16): both halves are its own, and
        // every head of the tile uses the same 16 pair indices c0...
        const int m = arow;
        const uint4* crow = reinterpret_cast<const uint4*>(args.rope_cos + static_cast<size_t>(m) * 64 + c0);
        const uint4* srow = reinterpret_cast<const uint4*>(args.rope_sin + static_cast<size_t>(m) * 64 + c0);
#pragma unroll 1
        for (int c = c0; c < BN; c += 64) {
          uint32_t va[16], vb[16];
          tmem_ld_x16(tbase + c, va);
          tmem_ld_x16(tbase + c + 32, vb);
          tmem_wait_ld();
          if (m >= args.M) continue;
          const int n0 = tb * BN + c;  // columns n0.. and n0 + 32..
          const int seg = n0 & ~63;
          uint32_t pa[8], pb[8];  // bf16(acc + bias), packed pairs
#pragma unroll
          for (int j = 0; j < 16; j += 2) {
            float a0 = __uint_as_float(va[j]), a1 = __uint_as_float(va[j + 1]);
            float b0 = __uint_as_float(vb[j]), b1 = __uint_as_float(vb[j + 1]);
            if (args.bias != nullptr) {
              a0 += bf16_to_f32(__ldg(args.bias + n0 + j));
              a1 += bf16_to_f32(__ldg(args.bias + n0 + j + 1));
              b0 += bf16_to_f32(__ldg(args.bias + n0 + 32 + j));
              b1 += bf16_to_f32(__ldg(args.bias + n0 + 33 + j));
            }
            pa[j / 2] = cvt_bf16x2(a0, a1);
            pb[j / 2] = cvt_bf16x2(b0, b1);
          }
          uint16_t* ya = args.y + static_cast<size_t>(m) * args.N + n0;
          if (seg < args.voff) {
            // this token's bf16 cos/sin at indices c0.. and c0 + 32.. (16-byte loads, L1-resident)
            uint32_t tc[16], ts[16];
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
              const uint4 cv = __ldg(crow + (q4 & 1) + (q4 >> 1) * 4);
              const uint4 sv = __ldg(srow + (q4 & 1) + (q4 >> 1) * 4);
              tc[4 * q4 + 0] = cv.x, tc[4 * q4 + 1] = cv.y, tc[4 * q4 + 2] = cv.z, tc[4 * q4 + 3] = cv.w;
              ts[4 * q4 + 0] = sv.x, ts[4 * q4 + 1] = sv.y, ts[4 * q4 + 2] = sv.z, ts[4 * q4 + 3] = sv.w;
            }
            uint32_t oa[8], ob[8];
#pragma unroll
            for (int p = 0; p < 8; ++p) {
              // pair p holds indices i = c0 + 2p, c0 + 2p + 1; each product and
              // the sums rounded to bf16 as rotate_head does
              const float f0 = bf16lo(pa[p]), f1 = bf16hi(pa[p]);  // first
              const float s0 = bf16lo(pb[p]), s1 = bf16hi(pb[p]);  // second
              const float cf0 = bf16lo(tc[p]), cf1 = bf16hi(tc[p]), cs0 = bf16lo(tc[8 + p]), cs1 = bf16hi(tc[8 + p]);
              const float sf0 = bf16lo(ts[p]), sf1 = bf16hi(ts[p]), ss0 = bf16lo(ts[8 + p]), ss1 = bf16hi(ts[8 + p]);
              const uint32_t left = cvt_bf16x2(f0 * cf0, f1 * cf1);
              const uint32_t right = cvt_bf16x2(-s0 * sf0, -s1 * sf1);
              const uint32_t right2 = cvt_bf16x2(f0 * ss0, f1 * ss1);
              const uint32_t left2 = cvt_bf16x2(s0 * cs0, s1 * cs1);
              oa[p] = cvt_bf16x2(bf16lo(left) + bf16lo(right), bf16hi(left) + bf16hi(right));
              ob[p] = cvt_bf16x2(bf16lo(left2) + bf16lo(right2), bf16hi(left2) + bf16hi(right2));
            }
            *reinterpret_cast<uint4*>(ya) = make_uint4(oa[0], oa[1], oa[2], oa[3]);
            *reinterpret_cast<uint4*>(ya + 8) = make_uint4(oa[4], oa[5], oa[6], oa[7]);
            *reinterpret_cast<uint4*>(ya + 32) = make_uint4(ob[0], ob[1], ob[2], ob[3]);
            *reinterpret_cast<uint4*>(ya + 40) = make_uint4(ob[4], ob[5], ob[6], ob[7]);
          } else {
            *reinterpret_cast<uint4*>(ya) = make_uint4(pa[0], pa[1], pa[2], pa[3]);
            *reinterpret_cast<uint4*>(ya + 8) = make_uint4(pa[4], pa[5], pa[6], pa[7]);
            *reinterpret_cast<uint4*>(ya + 32) = make_uint4(pb[0], pb[1], pb[2], pb[3]);
            *reinterpret_cast<uint4*>(ya + 40) = make_uint4(pb[4], pb[5], pb[6], pb[7]);
            // transposed copy: lanes hold consecutive tokens, so each column's store is contiguous
            uint16_t* vta = args.vt + static_cast<size_t>(n0 - args.voff) * args.M + m;
#pragma unroll
            for (int j = 0; j < 16; j += 2) {
              vta[static_cast<size_t>(j) * args.M] = static_cast<uint16_t>(pa[j / 2] & 0xFFFFu);
              vta[static_cast<size_t>(j + 1) * args.M] = static_cast<uint16_t>(pa[j / 2] >> 16);
              vta[static_cast<size_t>(j + 32) * args.M] = static_cast<uint16_t>(pb[j / 2] & 0xFFFFu);
              vta[static_cast<size_t>(j + 33) * args.M] = static_cast<uint16_t>(pb[j / 2] >> 16);
            }
          }
        }
      } else if (!SWAP && args.mode == 4) {
        // logits = (2 acc - esq) / d_scale * exp(log_inv_T) + bias (_TiedCodebookHead),
        // evaluated as fmaf(2 s, acc, -c) with the argmax form's operands
        const float s2 = -__ldg(args.head_scal + 2);
        const int m = arow;
#pragma unroll 1
        for (int c = c0; c < BN; c += 32) {
          uint32_t v[16];
          tmem_ld_x16(tbase + c, v);
          const int n0 = tb * BN + c;
          float4 cv[4];
          const bool vec = args.vec_ok && n0 + 16 <= args.N;
          if (vec) {
#pragma unroll
            for (int j = 0; j < 4; ++j) cv[j] = __ldg(reinterpret_cast<const float4*>(args.head_c + n0 + 4 * j));
          }
          tmem_wait_ld();
          if (m >= args.M) continue;
          float* dst = args.y_f32 + static_cast<size_t>(m) * args.N + n0;
          if (vec) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              float4 l;
              l.x = fmaf(s2, __uint_as_float(v[4 * j + 0]), -cv[j].x);
              l.y = fmaf(s2, __uint_as_float(v[4 * j + 1]), -cv[j].y);
              l.z = fmaf(s2, __uint_as_float(v[4 * j + 2]), -cv[j].z);
              l.w = fmaf(s2, __uint_as_float(v[4 * j + 3]), -cv[j].w);
              *reinterpret_cast<float4*>(dst + 4 * j) = l;
            }
          } else {
            for (int j = 0; j < 16 && n0 + j < args.N; ++j)
              dst[j] = fmaf(s2, __uint_as_float(v[j]), -__ldg(args.head_c + n0 + j));
          }
        }
      } else if (!SWAP && args.mode == 3) {
        // val = alpha * X + beta * (acc + bias), scattered to the real row
        const long long m = arow < args.M ? args.map.real_row(arow) : -1;
        const ConvEpilogue& ep = args.conv;
#pragma unroll 1
        for (int c = c0; c < BN; c += 32) {
          uint32_t v[16];
          tmem_ld_x16(tbase + c, v);
          const int n0 = tb * BN + c;
          const size_t o = static_cast<size_t>(m < 0 ? 0 : m) * args.N + n0;
          const bool vec = m >= 0 && args.vec_ok && n0 + 16 <= args.N;
          // issue this chunk's global reads before waiting for the tensor-memory load
          float4 xv[4], rv[4], av[4], bv[4];
          if (vec) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              xv[j] = make_float4(0.f, 0.f, 0.f, 0.f);
              if (ep.x_f32 != nullptr) {
                xv[j] = *reinterpret_cast<const float4*>(ep.x_f32 + o + 4 * j);
              } else if (ep.x_bf16 != nullptr) {
                const uint2 h = *reinterpret_cast<const uint2*>(ep.x_bf16 + o + 4 * j);
                xv[j] = make_float4(bf16lo(h.x), bf16hi(h.x), bf16lo(h.y), bf16hi(h.y));
              }
              rv[j] = ep.resid != nullptr ? *reinterpret_cast<const float4*>(ep.resid + o + 4 * j)
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
              av[j] = ep.acc_f32 != nullptr ? *reinterpret_cast<const float4*>(ep.acc_f32 + o + 4 * j)
                                            : make_float4(0.f, 0.f, 0.f, 0.f);
              bv[j] = ep.bias != nullptr ? __ldg(reinterpret_cast<const float4*>(ep.bias + n0 + 4 * j))
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
            }
          }
          tmem_wait_ld();
          if (m < 0) continue;
          if (vec) {
            // 16-byte accesses (N % 4 == 0 and every buffer 16-byte aligned)
#pragma unroll
            for (int j4 = 0; j4 < 4; ++j4) {
              const int j = 4 * j4;
              const float4 x = xv[j4], b = bv[j4];
              float4 val;
              val.x = fmaf(ep.alpha, x.x, ep.beta * (__uint_as_float(v[j]) + b.x));
              val.y = fmaf(ep.alpha, x.y, ep.beta * (__uint_as_float(v[j + 1]) + b.y));
              val.z = fmaf(ep.alpha, x.z, ep.beta * (__uint_as_float(v[j + 2]) + b.z));
              val.w = fmaf(ep.alpha, x.w, ep.beta * (__uint_as_float(v[j + 3]) + b.w));
              if (ep.out_f32 != nullptr) *reinterpret_cast<float4*>(ep.out_f32 + o + j) = val;
              if (ep.out_bf16 != nullptr)
                *reinterpret_cast<uint2*>(ep.out_bf16 + o + j) =
                    make_uint2(pack_bf16x2(val.x, val.y), pack_bf16x2(val.z, val.w));
              if (ep.resid != nullptr) {
                float4 r = rv[j4];
                r.x -= val.x;
                r.y -= val.y;
                r.z -= val.z;
                r.w -= val.w;
                *reinterpret_cast<float4*>(ep.resid + o + j) = r;
              }
              if (ep.acc_f32 != nullptr) {
                float4 a = av[j4];
                a.x += val.x;
                a.y += val.y;
                a.z += val.z;
                a.w += val.w;
                *reinterpret_cast<float4*>(ep.acc_f32 + o + j) = a;
              }
            }
            continue;
          }
#pragma unroll 1
          for (int j = 0; j < 16; ++j) {
            const int n = n0 + j;
            if (n >= args.N) break;
            const float cb = __uint_as_float(v[j]) + (ep.bias != nullptr ? __ldg(ep.bias + n) : 0.f);
            float x = 0.f;
            if (ep.x_f32 != nullptr)
              x = ep.x_f32[o + j];
            else if (ep.x_bf16 != nullptr)
              x = bf16_to_f32(ep.x_bf16[o + j]);
            const float val = fmaf(ep.alpha, x, ep.beta * cb);
            if (ep.out_f32 != nullptr) ep.out_f32[o + j] = val;
            if (ep.out_bf16 != nullptr) ep.out_bf16[o + j] = f32_to_bf16(val);
            if (ep.resid != nullptr) ep.resid[o + j] -= val;
            if (ep.acc_f32 != nullptr) ep.acc_f32[o + j] += val;
          }
        }
      } else
#pragma unroll 1
      for (int c = c0; c < BN; c += 32) {
        uint32_t v[16];
        tmem_ld_x16(tbase + c, v);
        // non-swapped rows: issue the bias and residual reads before waiting for the TMEM load
        const int n0 = tb * BN + c;
        const bool vrow = !SWAP && arow < args.M && args.vec_ok && n0 + 16 <= args.N;
        const size_t o = static_cast<size_t>(arow) * args.N + n0;
        uint4 h0 = make_uint4(0u, 0u, 0u, 0u), h1 = h0, bb0 = h0, bb1 = h0;
        if (vrow) {
          if (args.mode == 2) {
            h0 = *reinterpret_cast<const uint4*>(args.y + o);
            h1 = *reinterpret_cast<const uint4*>(args.y + o + 8);
          }
          if (args.bias != nullptr) {
            bb0 = __ldg(reinterpret_cast<const uint4*>(args.bias + n0));
            bb1 = __ldg(reinterpret_cast<const uint4*>(args.bias + n0 + 8));
          }
        }
        tmem_wait_ld();
        if (!SWAP) {
          // arow = token m, columns = outputs n
          const int m = arow;
          if (m < args.M) {
            float f[16];
            if (vrow) {
              const uint32_t bp[8] = {bb0.x, bb0.y, bb0.z, bb0.w, bb1.x, bb1.y, bb1.z, bb1.w};
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                f[2 * j] = __uint_as_float(v[2 * j]) + bf16lo(bp[j]);
                f[2 * j + 1] = __uint_as_float(v[2 * j + 1]) + bf16hi(bp[j]);
              }
            } else {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int n = n0 + j;
                float acc = __uint_as_float(v[j]);
                if (args.bias != nullptr && n < args.N) acc += bf16_to_f32(__ldg(args.bias + n));
                f[j] = acc;
              }
            }
            if (args.mode == 2) {
              // residual add (decoder.zig:310-313): y = bf16(y + bf16(acc + bias))
#pragma unroll
              for (int j = 0; j < 16; j += 2) {
                const uint32_t r = cvt_bf16x2(f[j], f[j + 1]);
                f[j] = bf16lo(r);
                f[j + 1] = bf16hi(r);
              }
              if (vrow) {
                const uint32_t hp[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  f[2 * j] += bf16lo(hp[j]);
                  f[2 * j + 1] += bf16hi(hp[j]);
                }
              } else {
                for (int j = 0; j < 16; ++j)
                  if (n0 + j < args.N) f[j] += bf16_to_f32(args.y[o + j]);
              }
            }
            if (args.y_f32 != nullptr) {
              for (int j = 0; j < 16; ++j)
                if (n0 + j < args.N) args.y_f32[o + j] = f[j];
            } else if (args.vec_ok && n0 + 16 <= args.N) {
              uint4 w0, w1;
              w0.x = cvt_bf16x2(f[0], f[1]);
              w0.y = cvt_bf16x2(f[2], f[3]);
              w0.z = cvt_bf16x2(f[4], f[5]);
              w0.w = cvt_bf16x2(f[6], f[7]);
              w1.x = cvt_bf16x2(f[8], f[9]);
              w1.y = cvt_bf16x2(f[10], f[11]);
              w1.z = cvt_bf16x2(f[12], f[13]);
              w1.w = cvt_bf16x2(f[14], f[15]);
              *reinterpret_cast<uint4*>(args.y + o) = w0;
              *reinterpret_cast<uint4*>(args.y + o + 8) = w1;
            } else {
              for (int j = 0; j < 16; ++j)
                if (n0 + j < args.N) args.y[o + j] = f32_to_bf16(f[j]);
            }
          }
        } else {
          // arow = output n, columns = tokens m
          const int n = arow;
          if (n < args.N && ksplit > 1) {
            // split-K: this split's f32 partial sums (bias and output in linear_ksplit_reduce_kernel)
            float* pp = args.part + static_cast<size_t>(unit % ksplit) * args.M * args.N + n;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int m = tb * BN + c + j;
              if (m < args.M) pp[static_cast<size_t>(m) * args.N] = __uint_as_float(v[j]);
            }
          } else if (n < args.N) {
            const float bv = args.bias != nullptr ? bf16_to_f32(__ldg(args.bias + n)) : 0.f;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int m = tb * BN + c + j;
              if (m < args.M) {
                float acc = __uint_as_float(v[j]) + bv;
                const size_t o = static_cast<size_t>(m) * args.N + n;
                if (args.mode == 2) acc = bf16_to_f32(f32_to_bf16(acc)) + bf16_to_f32(args.y[o]);
                if (args.y_f32 != nullptr)
                  args.y_f32[o] = acc;
                else
                  args.y[o] = f32_to_bf16(acc);
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR)
          mbar_arrive_cluster(mapa_shared(smem_u32(&S.tempty[b]), 0));  // the leader's barrier
        else
          mbar_arrive(&S.tempty[b]);
      }
      ++acc_it;
    }
    if (!ok) abort_all();
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  // a pair's partner may still read this CTA's shared memory (the leader's
  // MMAs) or arrive on its barriers until both are done
  if constexpr (PAIR) cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem, Cfg::TMEM_COLS);
    else
      tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

template <int BN, bool SWAP, bool PAIR>
constexpr size_t linear_smem_bytes() {
  static_assert(sizeof(GemmSmem<BN, PAIR>) + 1024 <= 232448, "GEMM shared memory budget");
  return sizeof(GemmSmem<BN, PAIR>) + 1024;
}

// Sets the dynamic shared-memory opt-in of one instantiation on the current
// device (once per device).
template <int BN, bool SWAP, bool PAIR>
cudaError_t linear_prepare() {
  static DeviceFlags attr_set;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (attr_set.test(dev)) return cudaSuccess;
  e = cudaFuncSetAttribute(linear_bf16_kernel<BN, SWAP, PAIR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(linear_smem_bytes<BN, SWAP, PAIR>()));
  if (e == cudaSuccess) attr_set.set(dev);
  return e;
}

cudaLaunchAttribute pair_cluster_attr() {
  cudaLaunchAttribute at{};
  at.id = cudaLaunchAttributeClusterDimension;
  at.val.clusterDim.x = 2;
  at.val.clusterDim.y = 1;
  at.val.clusterDim.z = 1;
  return at;
}

template <int BN, bool SWAP, bool PAIR>
cudaError_t launch_linear(const CUtensorMap& tmA, const CUtensorMap& tmB, const LinearArgs& a, int grid,
                          cudaStream_t stream) {
  cudaError_t e = linear_prepare<BN, SWAP, PAIR>();
  if (e != cudaSuccess) return e;
  constexpr size_t smem = linear_smem_bytes<BN, SWAP, PAIR>();
  return launch_pdl(linear_bf16_kernel<BN, SWAP, PAIR>, dim3(grid), dim3(THREADS), smem, stream, PAIR ? 2 : 1, tmA,
                    tmB, a);
}

// How many 2-CTA clusters of the 256-wide pair kernel fit at once (cluster
// placement can leave SMs idle); cached per device, 0 if none.
int max_pairs_linear(int num_sms) {
  static std::atomic<int> cached[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  const int known = cached[dev].load(std::memory_order_relaxed);
  if (known != 0) return known > 0 ? known : 0;
  int n = 0;
  if (linear_prepare<256, false, true>() == cudaSuccess) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(2 * (num_sms / 2));
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = linear_smem_bytes<256, false, true>();
    cudaLaunchAttribute at[1] = {pair_cluster_attr()};
    cfg.attrs = at;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, linear_bf16_kernel<256, false, true>, &cfg) != cudaSuccess) n = 0;
  }
  cudaGetLastError();
  const int v = n > 0 ? std::min(n, num_sms / 2) : -1;
  cached[dev].store(v, std::memory_order_relaxed);  // every thread computes the same value
  return v > 0 ? v : 0;
}

// Tile shape of a non-swapped GEMM with `rows` output rows and `cols` output
// columns (mode 1: cols = F, each tile holding bn/2 gate and bn/2 up columns).
// CTA pairs of 256-wide tiles when their tiles fill every pair; otherwise one
// CTA per tile with the widest tile that still fills the SMs.
struct GemmShape {
  int bn;
  bool pair;
};
GemmShape choose_shape(ncm_ctx* ctx, int64_t rows, int64_t cols, int mode) {
  const int pairs = max_pairs_linear(ctx->num_sms);
  const int64_t col_tiles_256 = mode == 1 ? cols / 128 : ceil_div(cols, 256);
  if (pairs > 0 && ceil_div(rows, 2 * BM) * col_tiles_256 >= pairs) return {256, true};
  const long long mt = ceil_div(rows, BM);
  if (mode == 1 || mt * ceil_div(cols, 256) >= ctx->num_sms) return {256, false};
  if (mt * ceil_div(cols, 128) >= ctx->num_sms) return {128, false};
  return {64, false};
}

// Builds the tensor maps for shape `sh` (A: [a_rows, a_cols] with 128-row
// boxes; B: [b_rows, k_cols] with boxes of the rows one CTA loads; a_cols =
// k_cols except for the kernel-3 convolution, whose B holds three taps), fills
// the tile counts of `a` (a.M output rows, a.N output columns) and launches.
int launch_shape(ncm_ctx* ctx, const GemmShape& sh, const void* A, int64_t a_rows, int64_t a_cols, const void* B,
                 int64_t b_rows, int64_t k_cols, LinearArgs& a, KernelId kid, cudaStream_t stream) {
  const uint32_t b_box = (sh.pair || a.mode == 1) ? sh.bn / 2 : sh.bn;
  CUtensorMap tmA, tmB;
  if (!make_tmap_bf16_2d(&tmA, A, a_rows, a_cols, BM) || !make_tmap_bf16_2d(&tmB, B, b_rows, k_cols, b_box))
    return ncm_fail(NCM_EINVAL, "gemm: tensor map encoding failed (rows=%lld K=%lld N=%lld)", (long long)a.M,
                    (long long)k_cols, (long long)a.N);
  a.tiles_a = ceil_div(a.M, sh.pair ? 2 * BM : BM);
  a.tiles_b = a.mode == 1 ? static_cast<int>(a.F / (sh.bn / 2)) : ceil_div(a.N, sh.bn);
  // keep the smaller operand L2-resident: walk the tiles of the larger one slowly
  const double a_bytes = double(a_rows) * a_cols * 2, b_bytes = double(b_rows) * k_cols * 2;
  a.a_fast = a_bytes <= b_bytes ? 1 : 0;
  const int tiles = a.tiles_a * a.tiles_b;
  int grid;
  if (sh.pair)
    grid = 2 * std::min(tiles, max_pairs_linear(ctx->num_sms));
  else
    grid = std::min(tiles, ctx->num_sms);
  cudaError_t e;
  Launch _launch(ctx, kid, stream);
  if (sh.pair) {
    e = launch_linear<256, false, true>(tmA, tmB, a, grid, stream);
  } else {
    switch (sh.bn) {
      case 256: e = launch_linear<256, false, false>(tmA, tmB, a, grid, stream); break;
      case 128: e = launch_linear<128, false, false>(tmA, tmB, a, grid, stream); break;
      default: e = launch_linear<64, false, false>(tmA, tmB, a, grid, stream); break;
    }
  }
  if (e != cudaSuccess) return ncm_set_cuda_error(e);
  return NCM_OK;
}

// y[m][n] = bf16(sum_s part[s][m][n] + bias[n]) in split order (mode 2:
// y = bf16(y + bf16(sum + bias)); f32 outputs when y_f32 is given): the
// epilogue of the split-K skinny GEMM, one thread per output.
__global__ void __launch_bounds__(256) linear_ksplit_reduce_kernel(const float* __restrict__ part, int ksplit,
                                                                   int M, int N, const uint16_t* __restrict__ bias,
                                                                   uint16_t* __restrict__ y, float* __restrict__ y_f32,
                                                                   int mode) {
  pdl_wait();
  pdl_launch_dependents();
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long MN = static_cast<long long>(M) * N;
  if (i >= MN) return;
  float acc = part[i];
  for (int s = 1; s < ksplit; ++s) acc += part[s * MN + i];
  if (bias != nullptr) acc += bf16_to_f32(__ldg(bias + i % N));
  if (mode == 2) acc = bf16_to_f32(f32_to_bf16(acc)) + bf16_to_f32(y[i]);
  if (y_f32 != nullptr)
    y_f32[i] = acc;
  else
    y[i] = f32_to_bf16(acc);
}

// The context's split-K partial buffer, grown on demand (freeing the old one
// waits for the device, so no launch still uses it).
float* ksplit_buffer(ncm_ctx* ctx, size_t bytes) {
  if (bytes <= ctx->kpart_bytes) return ctx->kpart;
  if (ctx->kpart != nullptr) {
    cudaFree(ctx->kpart);
    ctx->kpart = nullptr;
    ctx->kpart_bytes = 0;
  }
  const size_t want = std::max<size_t>(bytes, size_t(8) << 20);
  if (cudaMalloc(&ctx->kpart, want) != cudaSuccess) {
    cudaGetLastError();
    ctx->kpart = nullptr;
    return nullptr;
  }
  ctx->kpart_bytes = want;
  return ctx->kpart;
}

}  // namespace

int linear_bf16(ncm_ctx* ctx, const uint16_t* x, const uint16_t* w, const uint16_t* bias, uint16_t* y, float* y_f32,
                int64_t M, int64_t K, int64_t N, cudaStream_t stream) {
  return linear_bf16_ex(ctx, x, w, bias, y, y_f32, M, K, N, stream, 0, 0);
}

int linear_bf16_ex(ncm_ctx* ctx, const uint16_t* x, const uint16_t* w, const uint16_t* bias, uint16_t* y,
                   float* y_f32, int64_t M, int64_t K, int64_t N, cudaStream_t stream, int mode, int64_t F) {
  if (mode == 1 && (M <= 64 || F % 128 != 0 || N != 2 * F))
    return ncm_fail(NCM_EINVAL, "linear: fused SwiGLU needs M > 64, F %% 128 == 0, N == 2F");
  LinearArgs a{};
  a.taps = 1;
  a.mode = mode;
  a.F = static_cast<int>(F);
  a.bias = bias;
  a.y = y;
  a.y_f32 = y_f32;
  a.err = ctx->d_err;
  a.M = static_cast<int>(M);
  a.N = static_cast<int>(N);
  a.K = static_cast<int>(K);
  a.vec_ok = (N % 8 == 0) && ((reinterpret_cast<uintptr_t>(y) & 15) == 0) &&
             ((reinterpret_cast<uintptr_t>(bias) & 15) == 0);
  if (M > 64)
    return launch_shape(ctx, choose_shape(ctx, M, mode == 1 ? F : N, mode), x, M, K, w, N, K, a, KID_LINEAR, stream);
  // Skinny problems (decode-time GEMV shapes) run swapped: W is the 128-row
  // MMA operand and the tokens the narrow side
  const int bn = M <= 16 ? 16 : (M <= 32 ? 32 : 64);
  CUtensorMap tmA, tmB;
  if (!make_tmap_bf16_2d(&tmA, w, N, K, BM) || !make_tmap_bf16_2d(&tmB, x, M, K, bn))
    return ncm_fail(NCM_EINVAL, "linear: tensor map encoding failed (M=%lld K=%lld N=%lld)", (long long)M,
                    (long long)K, (long long)N);
  a.tiles_a = ceil_div(N, BM);
  a.tiles_b = ceil_div(M, bn);
  a.a_fast = 1;
  // Few tiles (decode-time GEMV shapes): split K so that about one unit per SM
  // streams its share of W, each split at least four 64-wide k-chunks; f32
  // partials, summed in split order by linear_ksplit_reduce_kernel (the sum
  // order differs from one accumulator's: within the f32-accumulation bar).
  const int nk = ceil_div(K, BK);
  const int tiles = a.tiles_a * a.tiles_b;
  a.ksplit = 1;
  if (mode == 0 || mode == 2) {
    const int want = std::min(ctx->num_sms / std::max(tiles, 1), nk / 4);
    if (want >= 3) {  // at least three times the CTAs, or the extra reduce pass does not pay
      a.nk_split = ceil_div(nk, want);
      a.ksplit = ceil_div(nk, a.nk_split);
    }
  }
  if (a.ksplit > 1) {
    a.part = ksplit_buffer(ctx, sizeof(float) * a.ksplit * static_cast<size_t>(M) * N);
    if (a.part == nullptr) return ncm_fail(NCM_ENOMEM, "linear: split-K buffer allocation failed");
  }
  const int grid = std::min(tiles * a.ksplit, ctx->num_sms);
  cudaError_t e;
  Launch _launch(ctx, KID_LINEAR, stream);
  switch (bn) {
    case 16: e = launch_linear<16, true, false>(tmA, tmB, a, grid, stream); break;
    case 32: e = launch_linear<32, true, false>(tmA, tmB, a, grid, stream); break;
    default: e = launch_linear<64, true, false>(tmA, tmB, a, grid, stream); break;
  }
  if (e != cudaSuccess) return ncm_set_cuda_error(e);
  if (a.ksplit > 1) {
    const long long mn = M * N;
    NCM_CUDA_TRY(launch_pdl(linear_ksplit_reduce_kernel, dim3(static_cast<unsigned>((mn + 255) / 256)), dim3(256), 0,
                            stream, 1, static_cast<const float*>(a.part), a.ksplit, static_cast<int>(M),
                            static_cast<int>(N), bias, y, y_f32, mode));
  }
  return NCM_OK;
}

int linear_qkv_rope(ncm_ctx* ctx, const uint16_t* x, const uint16_t* w, const uint16_t* bias, uint16_t* qkv,
                    uint16_t* vt, const uint16_t* cos_bf, const uint16_t* sin_bf, int64_t M, int64_t K, int64_t N,
                    int64_t voff, cudaStream_t stream) {
  if (M <= 64 || N % 64 != 0 || voff % 64 != 0 || voff > N)
    return ncm_fail(NCM_EINVAL, "qkv projection: fused RoPE needs M > 64 and head-aligned widths");
  LinearArgs a{};
  a.mode = 5;
  a.taps = 1;
  a.bias = bias;
  a.y = qkv;
  a.err = ctx->d_err;
  a.M = static_cast<int>(M);
  a.N = static_cast<int>(N);
  a.K = static_cast<int>(K);
  a.rope_cos = cos_bf;
  a.rope_sin = sin_bf;
  a.vt = vt;
  a.voff = static_cast<int>(voff);
  a.vec_ok = 1;
  return launch_shape(ctx, choose_shape(ctx, M, N, 5), x, M, K, w, N, K, a, KID_LINEAR, stream);
}

int tied_head_logits_gemm(ncm_ctx* ctx, const uint16_t* z, const uint16_t* codebook, const float* c,
                          const float* scal, float* logits, int64_t T, int64_t d, int64_t K, cudaStream_t stream) {
  LinearArgs a{};
  a.mode = 4;
  a.taps = 1;
  a.err = ctx->d_err;
  a.M = static_cast<int>(T);
  a.N = static_cast<int>(K);
  a.K = static_cast<int>(d);
  a.y_f32 = logits;
  a.head_c = c;
  a.head_scal = scal;
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  a.vec_ok = K % 4 == 0 && al(logits) && al(c);
  return launch_shape(ctx, choose_shape(ctx, T, K, 4), z, T, d, codebook, K, d, a, KID_LINEAR, stream);
}

int conv3_gemm(ncm_ctx* ctx, const uint16_t* a_pad, const uint16_t* w_pack, const SegMap& map, int64_t dp,
               int64_t width, const ConvEpilogue& ep, cudaStream_t stream) {
  const int64_t Mp = map.padded_rows();
  if (dp % BK != 0 || width <= 0 || Mp <= 0)
    return ncm_fail(NCM_EINVAL, "conv: padded width %lld must be a multiple of 64", (long long)dp);
  LinearArgs a{};
  a.mode = 3;
  a.err = ctx->d_err;
  a.M = static_cast<int>(Mp);
  a.N = static_cast<int>(width);
  a.K = static_cast<int>(3 * dp);
  a.taps = 3;
  a.nk_tap = static_cast<int>(dp / BK);
  a.conv = ep;
  a.map = map;
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  a.vec_ok = width % 4 == 0 && al(ep.x_f32) && al(ep.x_bf16) && al(ep.out_f32) && al(ep.out_bf16) &&
             al(ep.resid) && al(ep.acc_f32) && al(ep.bias);
  return launch_shape(ctx, choose_shape(ctx, Mp, width, 3), a_pad, Mp, dp, w_pack, width, 3 * dp, a, KID_CONV,
                      stream);
}

}  // namespace ncm
