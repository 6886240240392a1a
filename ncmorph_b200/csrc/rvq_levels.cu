// Every RVQ level of a small encode in one launch (R2 + R3 for small N).
//
// rvq_argmin_kernel runs one level per launch; when a problem has few row
// blocks (4,096 rows) its code range is split over CTAs
// and rvq_apply_kernel merges the splits and updates the residual in a
// second launch, so a 4-level encode is nine short launches whose fill and
// drain dominate. Here one cluster of C CTAs owns one 128-row block for all
// L levels:
//
//   CTA r of the cluster     code tiles [r * tpc, (r + 1) * tpc) of every level
//                            and residual columns [r * slice, (r + 1) * slice)
//   per level                distance GEMM of its tiles (tcgen05, TMA-staged,
//                            as rvq_argmin_kernel) -> per-row (distance, index)
//                            in its shared memory -> every CTA of the cluster
//                            reads all C partials through distributed shared
//                            memory, merges them (lowest distance, then lowest
//                            index: the same code as one CTA owning every
//                            tile) and updates its column slice of the f32
//                            residual and of the bf16 copy the next level's
//                            GEMM reads -> the next level's TMA loads wait
//                            until every CTA of the cluster has written its
//                            slice
//
// Hand-offs are cluster-scope mbarriers: each CTA's epilogue warps arrive on
// every CTA's "partials ready" barrier (double-buffered by level parity), and
// each CTA's update warps on every CTA's "level ready" barrier, which the TMA
// producer waits on. Every wait is bounded. The arithmetic of each row is
// the one of rvq_argmin_kernel + rvq_apply_kernel (or the fused update):
// codes and residuals are bit-identical to the per-level launches.
//
// Warp roles (448 threads): 0 TMA, 1 TMEM + MMA, 2-5 argmin epilogue (one
// thread per row), 6-13 merge + slice update (16 rows each).
#include <algorithm>
#include <cfloat>
#include <climits>
#include <cmath>

#include "internal.h"
#include "ptx.cuh"

namespace ncm {
namespace {

constexpr int LV_BM = 128;
constexpr int LV_BN = 256;
constexpr int LV_BK = 64;
constexpr int LV_STAGES = 4;
constexpr int LV_UPD_WARPS = 8;
constexpr int LV_UPD_ROWS = LV_BM / LV_UPD_WARPS;
constexpr int LV_THREADS = 64 + 128 + 32 * LV_UPD_WARPS;
constexpr int LV_A_BYTES = LV_BM * LV_BK * 2;
constexpr int LV_B_BYTES = LV_BN * LV_BK * 2;
constexpr uint32_t LV_TMEM_COLS = 2 * LV_BN;
constexpr int LV_MAX_CLUSTER = 8;  // portable cluster size

struct __align__(1024) LevelsSmem {
  uint8_t a[LV_STAGES][LV_A_BYTES];
  uint8_t b[LV_STAGES][LV_B_BYTES];
  float csq[4][LV_BN];     // per epilogue warp: ||e||^2 of the current code tile
  int2 xch[2][LV_BM];      // per level parity: (distance bits, index) of this CTA's tiles, per row
  uint64_t full[LV_STAGES];
  uint64_t empty[LV_STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t xfull[2];       // partials of every CTA of the cluster written (count C x 4)
  uint64_t lready;         // every CTA's slice of the next level's rows written (count C x 8)
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};
constexpr size_t LEVELS_SMEM = sizeof(LevelsSmem) + 1024;
static_assert(LEVELS_SMEM <= 232448, "shared memory budget");

struct LevelsArgs {
  const float* sqnorms;         // [L, K]
  int32_t* codes;               // [L, N]
  const uint16_t* x;            // level-0 rows, bf16 [N, D]
  float* resid;                 // f32 residual [N, D]
  uint16_t* shadow;             // bf16 copy of the residual: the GEMM operand of levels >= 1
  const uint16_t* codebooks;    // [L, K, D]
  int* err;
  int N, D, K, L;
  int code_tiles, tpc;          // code tiles per level, tiles per CTA
  int slice;                    // residual columns per CTA (multiple of 8)
  int keep_resid;               // the last level also updates resid
  uint16_t* recon;              // bf16 [N, D] reconstruction (REG kernels; may be null)
  // REG kernels: each CTA's slice is k-chunk `rank` and every k-chunk of a
  // level's code tile stays in the stage ring until the level's updates are
  // done, so a chosen codeword's slice is read from the owning CTA's shared
  // memory (distributed shared memory) instead of L2
  int gather_smem;
};

__device__ __forceinline__ void lv_abort(volatile int* abort_flag, int* err) {
  *abort_flag = 1;
  atomicOr(err, kErrWaitTimeout);
}

// One cluster per 128-row block: grid = row_blocks * C, cluster dims (C, 1, 1).
// REG: the CTA's residual slice (16 rows x at most 64 columns per update
// warp) stays in registers across the levels, next to the f32 sum of the
// chosen codewords, which becomes the bf16 reconstruction after the last
// level (the decode kernel's sum, in the same order); otherwise the residual
// lives in global memory and a decode launch follows.
template <bool REG>
__global__ void __launch_bounds__(LV_THREADS, 1)
    rvq_levels_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmS,
                      const __grid_constant__ CUtensorMap tmB, const LevelsArgs args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  LevelsSmem& S = *reinterpret_cast<LevelsSmem*>(smem_raw + pad);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int C = static_cast<int>(cluster_nctarank());
  const int rank = static_cast<int>(cluster_ctarank());
  const int row0 = static_cast<int>(blockIdx.x / C) * LV_BM;
  const int nk = (args.D + LV_BK - 1) / LV_BK;
  const int t0 = rank * args.tpc;
  const int t1 = min(t0 + args.tpc, args.code_tiles);

  if (threadIdx.x == 0) {
    for (int s = 0; s < LV_STAGES; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&S.tfull[b], 1);
      mbar_init(&S.tempty[b], 4);
      mbar_init(&S.xfull[b], 4 * C);
    }
    mbar_init(&S.lready, LV_UPD_WARPS * C);
    mbar_init(&S.drain, 1);
    S.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&S.tmem_base, LV_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // every CTA's barriers exist before any remote arrival
  tc_fence_after();
  pdl_wait();
  pdl_launch_dependents();
  const uint32_t tmem = S.tmem_base;
  volatile int* abort_flag = &S.abort_flag;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      tma_prefetch_desc(&tmX);
      tma_prefetch_desc(&tmS);
      tma_prefetch_desc(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      bool issued[LV_STAGES];
      uint32_t issued_parity[LV_STAGES];
      for (int s = 0; s < LV_STAGES; ++s) issued[s] = false, issued_parity[s] = 0;
      bool ok = true;
      for (int l = 0; ok && l < args.L; ++l) {
        if (l > 0) {
          // the rows of this level were written by every CTA of the cluster
          if (!mbar_wait_cluster(&S.lready, (l - 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          fence_proxy_async_global();
        }
        const CUtensorMap* tmA = l == 0 ? &tmX : &tmS;
        for (int t = t0; ok && t < t1; ++t) {
          for (int kc = 0; kc < nk; ++kc) {
            if (!mbar_wait(&S.empty[stage], phase ^ 1u, abort_flag)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&S.full[stage], LV_A_BYTES + LV_B_BYTES);
            tma_load_2d(tmA, &S.full[stage], S.a[stage], kc * LV_BK, row0);
            tma_load_2d(&tmB, &S.full[stage], S.b[stage], kc * LV_BK, l * args.K + t * LV_BN);
            issued[stage] = true;
            issued_parity[stage] = phase;
            if (++stage == LV_STAGES) {
              stage = 0;
              phase ^= 1u;
            }
          }
        }
      }
      if (!ok) {
        lv_abort(abort_flag, args.err);
        for (int s = 0; s < LV_STAGES; ++s)
          if (issued[s]) mbar_wait(&S.full[s], issued_parity[s], nullptr);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      const uint32_t idesc = idesc_bf16_f32(LV_BM, LV_BN);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t acc_it = 0;
      bool ok = true;
      for (int l = 0; ok && l < args.L; ++l) {
        for (int t = t0; ok && t < t1; ++t) {
          const uint32_t b = acc_it & 1u;
          const uint32_t ap = (acc_it >> 1) & 1u;
          if (!mbar_wait(&S.tempty[b], ap ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t dt = tmem + b * LV_BN;
          for (int kc = 0; kc < nk; ++kc) {
            if (!mbar_wait(&S.full[stage], phase, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a0 = smem_u32(S.a[stage]);
            const uint32_t b0 = smem_u32(S.b[stage]);
#pragma unroll
            for (int k = 0; k < LV_BK / 16; ++k)
              tc_mma_f16(dt, smem_desc_k_sw128(a0 + k * 32), smem_desc_k_sw128(b0 + k * 32), idesc,
                         (kc | k) != 0 ? 1u : 0u);
            tc_commit(&S.empty[stage]);
            if (++stage == LV_STAGES) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (!ok) break;
          tc_commit(&S.tfull[b]);
          ++acc_it;
        }
      }
      if (!ok) {
        lv_abort(abort_flag, args.err);
        tc_commit(&S.drain);
        mbar_wait(&S.drain, 0, nullptr);
      }
    }
  }
  else if (warp < 6) {
    // -------------------------------------------------- argmin epilogue
    // The distance loop is rvq_argmin_kernel's: dist = fmaf(-2, acc, ||e||^2)
    // over 32 columns at a time, the row's first minimum kept (strict <).
    const int q = warp & 3;
    float* csq_s = S.csq[warp - 2];
    const int rl = q * 32 + lane;  // this thread's row of the block
    uint32_t acc_it = 0;
    bool ok = true;
    for (int l = 0; ok && l < args.L; ++l) {
      const float* csq_l = args.sqnorms + static_cast<size_t>(l) * args.K;
      float best = INFINITY;
      int bidx = t0 * LV_BN;
      for (int t = t0; t < t1; ++t) {
        const uint32_t b = acc_it & 1u;
        const uint32_t ap = (acc_it >> 1) & 1u;
#pragma unroll
        for (int j = lane; j < LV_BN; j += 32) {
          const int code = t * LV_BN + j;
          csq_s[j] = code < args.K ? __ldg(csq_l + code) : INFINITY;
        }
        __syncwarp();
        if (!__all_sync(0xffffffffu, mbar_wait(&S.tfull[b], ap, abort_flag))) {  // warp-uniform: TMEM loads follow
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tbase = tmem + (static_cast<uint32_t>(q * 32) << 16) + b * LV_BN;
#pragma unroll 1
        for (int c2 = 0; c2 < LV_BN; c2 += 64) {
          // two 32-column loads per wait: the epilogue is bound by tensor-memory
          // round trips when a level has one tile per CTA
          uint32_t v[2][32];
          tmem_ld_x32(tbase + c2, v[0]);
          tmem_ld_x32(tbase + c2 + 32, v[1]);
          tmem_wait_ld();
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int c = c2 + 32 * hh;
            const float4* cs4 = reinterpret_cast<const float4*>(csq_s + c);
            float m = INFINITY;
#pragma unroll
            for (int j4 = 0; j4 < 8; ++j4) {
              const float4 cv = cs4[j4];
              const float d0 = fmaf(-2.f, __uint_as_float(v[hh][4 * j4 + 0]), cv.x);
              const float d1 = fmaf(-2.f, __uint_as_float(v[hh][4 * j4 + 1]), cv.y);
              const float d2 = fmaf(-2.f, __uint_as_float(v[hh][4 * j4 + 2]), cv.z);
              const float d3 = fmaf(-2.f, __uint_as_float(v[hh][4 * j4 + 3]), cv.w);
              v[hh][4 * j4 + 0] = __float_as_uint(d0);
              v[hh][4 * j4 + 1] = __float_as_uint(d1);
              v[hh][4 * j4 + 2] = __float_as_uint(d2);
              v[hh][4 * j4 + 3] = __float_as_uint(d3);
              m = fminf(m, fminf(fminf(d0, d1), fminf(d2, d3)));
            }
            if (m < best) {  // strict: an equal distance from a lower code keeps its place
              int jj = 0;
#pragma unroll
              for (int j = 31; j >= 0; --j) jj = (__uint_as_float(v[hh][j]) == m) ? j : jj;
              best = m;
              bidx = t * LV_BN + c + jj;
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.tempty[b]);
        ++acc_it;
      }
      if (!ok) break;
      // publish this CTA's partial of the row; every CTA of the cluster reads it
      S.xch[l & 1][rl] = make_int2(__float_as_int(best), bidx);
      __syncwarp();  // the warp's writes precede lane 0's cluster-scope release below
      if (lane == 0)
        for (int p = 0; p < C; ++p) mbar_arrive_cluster(mapa_shared(smem_u32(&S.xfull[l & 1]), p));
    }
    if (!ok) lv_abort(abort_flag, args.err);
  } else {
    // ------------------------------------------- merge + slice update
    const int uw = warp - 6;
    const int c_lo = rank * args.slice;
    const int c_hi = min(c_lo + args.slice, args.D);
    const int nq = max((c_hi - c_lo) >> 2, 0);  // float4 chunks per row of this CTA's slice
    const int total = LV_UPD_ROWS * nq;
    const int rbase = row0 + uw * LV_UPD_ROWS;
    // REG: lane's chunk jj is idx = lane + 32 jj of the warp's rows x slice
    constexpr int NJ = REG ? 8 : 1;
    float4 r[NJ], qa[NJ];
    if constexpr (REG) {
#pragma unroll
      for (int jj = 0; jj < NJ; ++jj) {
        r[jj] = qa[jj] = make_float4(0.f, 0.f, 0.f, 0.f);
        const int idx = lane + 32 * jj;
        if (idx < total) {
          const int i = idx / nq;
          const int row = rbase + i;
          if (row < args.N) {
            const uint2 sv = *reinterpret_cast<const uint2*>(args.x + static_cast<size_t>(row) * args.D + c_lo +
                                                             (idx - i * nq) * 4);
            r[jj] = make_float4(bf16lo(sv.x), bf16hi(sv.x), bf16lo(sv.y), bf16hi(sv.y));
          }
        }
      }
    }
    bool ok = true;
    for (int l = 0; ok && l < args.L; ++l) {
      if (!__all_sync(0xffffffffu, mbar_wait_cluster(&S.xfull[l & 1], (l >> 1) & 1, abort_flag))) {
        ok = false;
        break;
      }
      // lanes 0-15: one row each; the C partials of the row, lowest distance
      // then lowest index (rvq_apply_kernel's merge)
      int code = -1;
      const int rl = uw * LV_UPD_ROWS + (lane & (LV_UPD_ROWS - 1));
      const int row = row0 + rl;
      if (lane < LV_UPD_ROWS) {
        const uint32_t xa = smem_u32(&S.xch[l & 1][rl]);
        int2 pv[LV_MAX_CLUSTER];
#pragma unroll
        for (int p = 0; p < LV_MAX_CLUSTER; ++p)
          if (p < C) pv[p] = ld_shared_cluster_v2(mapa_shared(xa, p));
        float bd = INFINITY;
        int bi = INT_MAX;
#pragma unroll
        for (int p = 0; p < LV_MAX_CLUSTER; ++p) {
          if (p < C) {
            const float d = __int_as_float(pv[p].x);
            if (d < bd || (d == bd && pv[p].y < bi)) bd = d, bi = pv[p].y;
          }
        }
        if (bi == INT_MAX) bi = pv[0].y;  // every distance was NaN/inf
        code = bi;
        if (row < args.N) {
          if (rank == 0) args.codes[static_cast<size_t>(l) * args.N + row] = code;
          if (code < 0 || code >= args.K) {
            atomicOr(args.err, kErrBadIndex);
            code = -1;
          }
        } else {
          code = -1;
        }
      }
      const bool last = l == args.L - 1;
      const uint16_t* cb = args.codebooks + static_cast<size_t>(l) * args.K * args.D;
      if constexpr (REG) {
        // resid -= e[code], q += e[code] on the registers; bf16(resid) for the
        // next level; after the last level the kept residual and bf16(q)
        // two passes of four chunks: each pass's codeword loads go out together
#pragma unroll
        for (int h0 = 0; h0 < NJ; h0 += 4) {
          uint2 ev[4];
          int cdj[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int idx = lane + 32 * (h0 + u);
            const int i = idx / max(nq, 1);
            cdj[u] = __shfl_sync(0xffffffffu, code, i & (LV_UPD_ROWS - 1));
            if (idx >= total) cdj[u] = -1;
            if (cdj[u] >= 0) {
              const int colin = (idx - i * nq) * 4;  // column inside the slice
              if (args.gather_smem) {
                // row (code % 256) of the owner's B tile, k-chunk `rank`: 128-byte
                // rows, 16-byte chunk j stored at j ^ (row % 8)
                const int owner = cdj[u] / LV_BN;
                const int crow = cdj[u] - owner * LV_BN;
                const int stage = (l * nk + rank) % LV_STAGES;
                const uint32_t a = smem_u32(S.b[stage]) + crow * 128 + ((((colin >> 3) ^ (crow & 7))) << 4) +
                                   (colin & 7) * 2;
                const int2 g = ld_shared_cluster_v2(mapa_shared(a, owner));
                ev[u] = make_uint2(static_cast<uint32_t>(g.x), static_cast<uint32_t>(g.y));
              } else {
                ev[u] = __ldg(reinterpret_cast<const uint2*>(cb + static_cast<size_t>(cdj[u]) * args.D + c_lo + colin));
              }
            }
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            if (cdj[u] < 0) continue;
            const int jj = h0 + u;
            const int idx = lane + 32 * jj;
            const int i = idx / nq;
            const size_t off = static_cast<size_t>(rbase + i) * args.D + c_lo + (idx - i * nq) * 4;
            const float e0 = bf16lo(ev[u].x), e1 = bf16hi(ev[u].x), e2 = bf16lo(ev[u].y), e3 = bf16hi(ev[u].y);
            r[jj].x -= e0;
            r[jj].y -= e1;
            r[jj].z -= e2;
            r[jj].w -= e3;
            qa[jj].x += e0;
            qa[jj].y += e1;
            qa[jj].z += e2;
            qa[jj].w += e3;
            if (!last) {
              *reinterpret_cast<uint2*>(args.shadow + off) =
                  make_uint2(pack_bf16x2(r[jj].x, r[jj].y), pack_bf16x2(r[jj].z, r[jj].w));
            } else {
              if (args.keep_resid) *reinterpret_cast<float4*>(args.resid + off) = r[jj];
              if (args.recon != nullptr)
                *reinterpret_cast<uint2*>(args.recon + off) =
                    make_uint2(pack_bf16x2(qa[jj].x, qa[jj].y), pack_bf16x2(qa[jj].z, qa[jj].w));
            }
          }
        }
      } else if (!last || args.keep_resid) {
        // this CTA's columns of the warp's 16 rows: resid = src - e[code]
        // (src = f32(x) at level 0, else resid), and bf16(resid) for the next
        // level; flat float4 chunks over the warp, four chunks' loads before
        // their stores
        constexpr int CH = 4;
#pragma unroll 1
        for (int base = 0; base < total; base += CH * 32) {
          float4 x4[CH];
          uint2 ev[CH];
          size_t off[CH];
          bool act[CH];
#pragma unroll
          for (int j = 0; j < CH; ++j) {
            const int idx = base + j * 32 + lane;
            const int i = idx / max(nq, 1);
            const int cd = __shfl_sync(0xffffffffu, code, i & (LV_UPD_ROWS - 1));
            act[j] = idx < total && cd >= 0;
            off[j] = 0;
            if (act[j]) {
              const int col = c_lo + (idx - i * nq) * 4;
              off[j] = static_cast<size_t>(rbase + i) * args.D + col;
              if (l == 0) {
                const uint2 sv = *reinterpret_cast<const uint2*>(args.x + off[j]);
                x4[j] = make_float4(bf16lo(sv.x), bf16hi(sv.x), bf16lo(sv.y), bf16hi(sv.y));
              } else {
                x4[j] = *reinterpret_cast<const float4*>(args.resid + off[j]);
              }
              ev[j] = __ldg(reinterpret_cast<const uint2*>(cb + static_cast<size_t>(cd) * args.D + col));
            }
          }
#pragma unroll
          for (int j = 0; j < CH; ++j) {
            if (act[j]) {
              float4 v = x4[j];
              v.x -= bf16lo(ev[j].x);
              v.y -= bf16hi(ev[j].x);
              v.z -= bf16lo(ev[j].y);
              v.w -= bf16hi(ev[j].y);
              *reinterpret_cast<float4*>(args.resid + off[j]) = v;
              if (!last)
                *reinterpret_cast<uint2*>(args.shadow + off[j]) =
                    make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
            }
          }
        }
      }
      if (!last) {
        // the next level's TMA loads read these rows: release them to the cluster
        fence_proxy_async_global();
        __syncwarp();
        if (lane == 0)
          for (int p = 0; p < C; ++p) mbar_arrive_cluster(mapa_shared(smem_u32(&S.lready), p));
      }
    }
    if (!ok) lv_abort(abort_flag, args.err);
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  // no CTA leaves while another may still read its partials or arrive on its barriers
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, LV_TMEM_COLS);
  }
}

}  // namespace
}  // namespace ncm

// ================================================================== host
namespace ncm {

bool rvq_levels_plan(int num_sms, int64_t N, int64_t D, int64_t K, int L, RvqLevelsPlan* out) {
  const int row_blocks = static_cast<int>(ceil_div(N, LV_BM));
  const int code_tiles = static_cast<int>(ceil_div(K, LV_BN));
  // Only where one level per launch would split the code range over CTAs
  // (few row blocks), and where every CTA of a cluster can hold a single code
  // tile: with several tiles per CTA the cluster has less tensor-core
  // parallelism per level than the split plan, which outweighs the saved
  // launches (one level's chain of TMA, MMA, argmin, exchange and update is
  // latency-bound at these sizes either way).
  if (L < 2 || row_blocks <= 0 || row_blocks * 2 > num_sms || D % 8 != 0) return false;
  if (code_tiles > LV_MAX_CLUSTER || static_cast<int64_t>(row_blocks) * code_tiles > num_sms) return false;
  out->row_blocks = row_blocks;
  out->cluster = code_tiles;
  out->tpc = 1;
  out->code_tiles = code_tiles;
  out->slice = static_cast<int>(ceil_div(ceil_div(D, code_tiles), 8) * 8);
  // 16 rows x slice / 4 float4 per update warp fit eight per lane
  out->reg = out->slice <= 64 ? 1 : 0;
  return true;
}

cudaError_t launch_rvq_levels(const RvqLevelsPlan& plan, const uint16_t* x, const uint16_t* codebooks,
                              const float* sqnorms, int L, int32_t* codes, float* resid, bool keep_resid,
                              uint16_t* shadow, uint16_t* recon, int* err, int64_t N, int64_t D, int64_t K,
                              cudaStream_t stream) {
  CUtensorMap tmX, tmS, tmB;
  if (!make_tmap_bf16_2d(&tmX, x, N, D, LV_BM) || !make_tmap_bf16_2d(&tmS, shadow, N, D, LV_BM) ||
      !make_tmap_bf16_2d(&tmB, codebooks, static_cast<uint64_t>(L) * K, D, LV_BN))
    return cudaErrorInvalidValue;
  static DeviceFlags attr_set[2];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (!attr_set[plan.reg].test(dev)) {
    e = cudaFuncSetAttribute(plan.reg ? rvq_levels_kernel<true> : rvq_levels_kernel<false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(LEVELS_SMEM));
    if (e != cudaSuccess) return e;
    attr_set[plan.reg].set(dev);
  }
  LevelsArgs a{};
  a.sqnorms = sqnorms;
  a.codes = codes;
  a.x = x;
  a.resid = resid;
  a.shadow = shadow;
  a.codebooks = codebooks;
  a.err = err;
  a.N = static_cast<int>(N);
  a.D = static_cast<int>(D);
  a.K = static_cast<int>(K);
  a.L = L;
  a.code_tiles = plan.code_tiles;
  a.tpc = plan.tpc;
  a.slice = plan.slice;
  a.keep_resid = keep_resid ? 1 : 0;
  a.recon = plan.reg ? recon : nullptr;
  a.gather_smem = (plan.reg && plan.tpc == 1 && plan.slice == LV_BK && ceil_div(D, LV_BK) <= LV_STAGES) ? 1 : 0;
  const dim3 grid(plan.row_blocks * plan.cluster);
  if (plan.reg)
    return launch_pdl(rvq_levels_kernel<true>, grid, dim3(LV_THREADS), LEVELS_SMEM, stream, plan.cluster, tmX, tmS,
                      tmB, a);
  return launch_pdl(rvq_levels_kernel<false>, grid, dim3(LV_THREADS), LEVELS_SMEM, stream, plan.cluster, tmX, tmS, tmB,
                    a);
}

}  // namespace ncm
