// Residual-vector-quantisation kernels (R1-R6).
//
// The per-level hot kernel, rvq_argmin_kernel, is the distance GEMM
//     dist[n,k] = ||e_k||^2 - 2 * bf16(r_n) . e_k
// on the 5th-generation tensor cores (tcgen05.mma, bf16 operands, f32
// accumulators in tensor memory) with the argmin folded into the epilogue, so
// the [N,K] distance matrix never leaves the SM. Operand tiles arrive by TMA
// into 128-byte-swizzled shared memory; a 4-stage mbarrier ring overlaps TMA,
// MMA and the argmin epilogue, and two 256-column TMEM accumulators let the
// epilogue of code tile t run while the MMA of tile t+1 proceeds.
//
// Warp roles (448 threads, one CTA per SM, persistent over work units):
//   warp 0     TMA producer (one elected lane)
//   warp 1     TMEM allocator + MMA issuer (one elected lane)
//   warps 2-5  argmin epilogue, one thread per accumulator row (TMEM lane)
//   warps 6-13 residual update: when a row block's codes are final they
//              apply r -= e[code] (f32) and write bf16(r) for the next level,
//              while the tensor cores already work on the next row block
//
// A work unit is (row block of 128 residuals, range of code tiles). When the
// rows alone cannot fill the GPU the code range is split and each split
// writes a (distance, index) partial per row. The splits are then merged by
// rvq_apply_kernel, which also applies the residual update over every SM, or,
// when no update follows, by the CTA that finishes a row block's last split.
// (A cooperative variant, in which every split's CTA waited for the row
// block's other splits and updated its own column slice, measured slower at
// every size from 1,024 to 8,192 rows: the update then ran at the end of the
// kernel on 8 warps per SM, with far less memory parallelism than the
// separate full-GPU apply launch.)
#include <algorithm>
#include <cfloat>
#include <climits>
#include <cmath>

#include "internal.h"
#include "ptx.cuh"

namespace ncm {
namespace {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int UPD_WARPS = 8;  // residual-update warps (rows split evenly among them)
constexpr int UPD_ROWS = BM / UPD_WARPS;
constexpr int THREADS = 64 + 128 + 32 * UPD_WARPS;
constexpr int A_BYTES = BM * BK * 2;
constexpr uint32_t TMEM_COLS = 2 * BN;

// Stage layout of one CTA. PAIR: the CTA holds half of each 256-code tile
// (its partner the other half), so a stage is half as large and six fit.
template <bool PAIR>
struct ArgminCfg {
  static constexpr int STAGES = PAIR ? 6 : 4;
  static constexpr int B_ROWS = PAIR ? BN / 2 : BN;
  static constexpr int B_TILE = B_ROWS * BK * 2;
  // bytes the leader's full barrier counts per stage (both CTAs' copies in a pair)
  static constexpr uint32_t STAGE_TX = PAIR ? 2u * (A_BYTES + B_TILE) : A_BYTES + B_TILE;
};

template <bool PAIR>
struct __align__(1024) ArgminSmem {
  static constexpr int STAGES = ArgminCfg<PAIR>::STAGES;
  uint8_t a[STAGES][A_BYTES];
  uint8_t b[STAGES][ArgminCfg<PAIR>::B_TILE];
  float csq[4][BN];  // per epilogue warp: ||e||^2 of the current code tile
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t drain;
  uint64_t upd_full[2];   // epilogue -> update warps: a row block's codes are in codes_s
  uint64_t upd_empty[2];  // update warps -> epilogue: codes_s slot free again
  uint64_t fix_arrive;    // split fixup: the 4 argmin warps published their partials
  uint64_t fix_done;      // split fixup: the arrival was counted, fix_last is set
  int codes_s[2][BM];
  int upd_rb[2];   // row block of each handoff; -1 ends the update warps' loop
  int fix_last;    // split fixup: this CTA finished the row block's last split
  uint32_t tmem_base;
  int abort_flag;
};
template <bool PAIR>
constexpr size_t argmin_smem_bytes() {
  return sizeof(ArgminSmem<PAIR>) + 1024;
}
static_assert(argmin_smem_bytes<false>() <= 232448 && argmin_smem_bytes<true>() <= 232448, "shared memory budget");

struct ArgminArgs {
  const float* csq;
  int32_t* codes;
  RvqPartial* part;
  int* err;
  int N, D, K;
  int splits, tiles_per_split, code_tiles, n_units;
  // fused residual update (splits == 1 only)
  int fuse;
  float* resid;
  const uint16_t* src_bf16;  // level input in bf16 (level 0), else null: read resid
  uint16_t* shadow;          // bf16(resid) for the next level, or null
  const uint16_t* codebook;
  // dist = fmaf(mul, acc, csq[k]); mul = -2 (RVQ) or *mul_dev when given (tied head)
  const float* mul_dev;
  // split fixup (splits > 1, no update): per row block arrival counters
  // (zero before the launch, zero again after it); the CTA that completes a
  // row block's last split merges the partials and writes the codes
  int* counters;
  // top-2 gap (the GAP instantiation only)
  float* gap;        // [N] relative gap, splits == 1
  const float* a2;   // [N] ||bf16(r)||^2
  float* part_d2;    // [splits, N] second-smallest distance of each split
};

// (second - best) / (||a||^2 + best): the top-2 gap relative to the best full
// squared distance (||r||^2 is the constant the GEMM distance leaves out).
__device__ __forceinline__ float rel_gap(float s1, float s2, float a2) {
  return (s2 - s1) / fmaxf(a2 + s1, 1e-30f);
}

__device__ __forceinline__ void raise_abort(volatile int* abort_flag, int* err) {
  *abort_flag = 1;
  atomicOr(err, kErrWaitTimeout);
}

// GAP: also track the second-smallest distance per row for the top-2 gap.
// PAIR: launched as clusters of 2 CTAs sharing each MMA (cta_group::2): a
// unit is then 256 rows (128 per CTA) and the even CTA issues the MMAs.
template <bool GAP, bool PAIR>
__global__ void __launch_bounds__(THREADS, 1)
    rvq_argmin_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const ArgminArgs args) {
  constexpr int STAGES = ArgminCfg<PAIR>::STAGES;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  ArgminSmem<PAIR>& S = *reinterpret_cast<ArgminSmem<PAIR>*>(smem_raw + pad);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nk = (args.D + BK - 1) / BK;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;  // 0 = leader (issues the pair's MMAs)
  const int cid = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int ncl = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  // unit -> first row this CTA owns, and the index of its 128-row block
  auto unit_rows = [&](int unit, int& rbase, int& rblock) {
    const int rb = unit / args.splits;
    rbase = PAIR ? rb * 2 * BM + static_cast<int>(rank) * BM : rb * BM;
    rblock = rbase / BM;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&S.tfull[b], 1);
      mbar_init(&S.tempty[b], PAIR ? 8 : 4);  // a pair's leader hears both CTAs' epilogues
      mbar_init(&S.upd_full[b], 4);
      mbar_init(&S.upd_empty[b], UPD_WARPS);
    }
    mbar_init(&S.drain, 1);
    mbar_init(&S.fix_arrive, 4);
    mbar_init(&S.fix_done, 1);
    S.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(&S.tmem_base, TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(&S.tmem_base, TMEM_COLS);
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
    raise_abort(abort_flag, args.err);
    if constexpr (PAIR) st_shared_cluster_u32(mapa_shared(smem_u32(&S.abort_flag), rank ^ 1u), 1u);
  };

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_parity[STAGES];
      bool issued[STAGES];
      for (int s = 0; s < STAGES; ++s) issued[s] = false, issued_parity[s] = 0;
      bool ok = true;
      for (int unit = cid; ok && unit < args.n_units; unit += ncl) {
        int rbase, rblock;
        unit_rows(unit, rbase, rblock);
        const int sp = unit - (unit / args.splits) * args.splits;
        const int t0 = sp * args.tiles_per_split;
        const int t1 = min(t0 + args.tiles_per_split, args.code_tiles);
        for (int t = t0; ok && t < t1; ++t) {
          for (int kc = 0; kc < nk; ++kc) {
            if (!mbar_wait(&S.empty[stage], phase ^ 1u, abort_flag)) {
              ok = false;
              break;
            }
            if constexpr (PAIR) {
              // both CTAs' copies complete on the leader's full barrier; the
              // leader posts the expected bytes of both
              if (rank == 0) mbar_arrive_expect_tx(&S.full[stage], ArgminCfg<PAIR>::STAGE_TX);
              const uint32_t fb = mapa_shared(smem_u32(&S.full[stage]), 0);
              tma_load_2d_pair(&tmA, fb, S.a[stage], kc * BK, rbase);
              tma_load_2d_pair(&tmB, fb, S.b[stage], kc * BK, t * BN + static_cast<int>(rank) * (BN / 2));
            } else {
              mbar_arrive_expect_tx(&S.full[stage], ArgminCfg<PAIR>::STAGE_TX);
              tma_load_2d(&tmA, &S.full[stage], S.a[stage], kc * BK, rbase);
              tma_load_2d(&tmB, &S.full[stage], S.b[stage], kc * BK, t * BN);
            }
            issued[stage] = true;
            issued_parity[stage] = phase;
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1u;
            }
          }
        }
      }
      if (!ok) {
        abort_all();
        // let every copy this thread issued land before the CTA exits (a
        // pair's follower cannot observe the leader's barrier: it waits a
        // fixed 20 us, far longer than any copy takes)
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
      // ------------------------------------------------ MMA issuer
      const uint32_t idesc = idesc_bf16_f32(PAIR ? 2 * BM : BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t acc_it = 0;
      bool ok = true;
      for (int unit = cid; ok && unit < args.n_units; unit += ncl) {
        const int sp = unit - (unit / args.splits) * args.splits;
        const int t0 = sp * args.tiles_per_split;
        const int t1 = min(t0 + args.tiles_per_split, args.code_tiles);
        for (int t = t0; ok && t < t1; ++t) {
          const uint32_t b = acc_it & 1u;
          const uint32_t ap = (acc_it >> 1) & 1u;
          if (!mbar_wait(&S.tempty[b], ap ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t dt = tmem + b * BN;
          for (int kc = 0; kc < nk; ++kc) {
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
                                (kc | k) != 0 ? 1u : 0u);
              else
                tc_mma_f16(dt, smem_desc_k_sw128(a0 + k * 32), smem_desc_k_sw128(b0 + k * 32), idesc,
                           (kc | k) != 0 ? 1u : 0u);
            }
            // the stage is free again in both CTAs of a pair
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
      }
      if (!ok) {
        abort_all();
        // wait for every MMA issued so far before TMEM is freed
        if constexpr (PAIR)
          tc_commit_pair(&S.drain, 0x1);
        else
          tc_commit(&S.drain);
        mbar_wait(&S.drain, 0, nullptr);
      }
    }
  } else if (warp < 6) {
    // -------------------------------------------------- argmin epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    float* csq_s = S.csq[warp - 2];
    const float mul = args.mul_dev != nullptr ? __ldg(args.mul_dev) : -2.f;
    uint32_t acc_it = 0;
    uint32_t uit = 0;     // units handed to the update warps
    uint32_t fix_ph = 0;  // phase of the split-fixup handshake barriers
    bool ok = true;
    for (int unit = cid; ok && unit < args.n_units; unit += ncl) {
      int rbase, rb;
      unit_rows(unit, rbase, rb);
      const int sp = unit - (unit / args.splits) * args.splits;
      const int t0 = sp * args.tiles_per_split;
      const int t1 = min(t0 + args.tiles_per_split, args.code_tiles);
      const int row = rbase + q * 32 + lane;
      float best = INFINITY;
      int bidx = t0 * BN;
      float s1 = INFINITY, s2 = INFINITY;  // GAP: smallest and second-smallest distance
      for (int t = t0; t < t1; ++t) {
        const uint32_t b = acc_it & 1u;
        const uint32_t ap = (acc_it >> 1) & 1u;
        // ||e||^2 of this tile's codes; codes past K get +inf so they never win
#pragma unroll
        for (int j = lane; j < BN; j += 32) {
          const int code = t * BN + j;
          csq_s[j] = code < args.K ? __ldg(args.csq + code) : INFINITY;
        }
        __syncwarp();
        if (!__all_sync(0xffffffffu, mbar_wait(&S.tfull[b], ap, abort_flag))) {  // warp-uniform: TMEM loads follow
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tbase = tmem + (static_cast<uint32_t>(q * 32) << 16) + b * BN;
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t v[32];
          tmem_ld_x32(tbase + c, v);
          tmem_wait_ld();
          const float4* cs4 = reinterpret_cast<const float4*>(csq_s + c);
          float m = INFINITY;
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4) {
            const float4 cv = cs4[j4];
            const float d0 = fmaf(mul, __uint_as_float(v[4 * j4 + 0]), cv.x);
            const float d1 = fmaf(mul, __uint_as_float(v[4 * j4 + 1]), cv.y);
            const float d2 = fmaf(mul, __uint_as_float(v[4 * j4 + 2]), cv.z);
            const float d3 = fmaf(mul, __uint_as_float(v[4 * j4 + 3]), cv.w);
            v[4 * j4 + 0] = __float_as_uint(d0);
            v[4 * j4 + 1] = __float_as_uint(d1);
            v[4 * j4 + 2] = __float_as_uint(d2);
            v[4 * j4 + 3] = __float_as_uint(d3);
            m = fminf(m, fminf(fminf(d0, d1), fminf(d2, d3)));
            if constexpr (GAP) {
              s2 = fminf(s2, fmaxf(s1, d0));
              s1 = fminf(s1, d0);
              s2 = fminf(s2, fmaxf(s1, d1));
              s1 = fminf(s1, d1);
              s2 = fminf(s2, fmaxf(s1, d2));
              s1 = fminf(s1, d2);
              s2 = fminf(s2, fmaxf(s1, d3));
              s1 = fminf(s1, d3);
            }
          }
          if (m < best) {  // strict: an equal distance from a lower code keeps its place
            int jj = 0;
#pragma unroll
            for (int j = 31; j >= 0; --j) jj = (__uint_as_float(v[j]) == m) ? j : jj;
            best = m;
            bidx = t * BN + c + jj;
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
      if (!ok) break;
      if (row < args.N) {
        if (args.splits == 1) {
          args.codes[row] = bidx;
          if constexpr (GAP) args.gap[row] = rel_gap(s1, s2, args.a2[row]);
        } else {
          args.part[static_cast<size_t>(sp) * args.N + row] = RvqPartial{best, bidx};
          if constexpr (GAP) args.part_d2[static_cast<size_t>(sp) * args.N + row] = s2;
        }
      }
      if (args.splits > 1) {
        if (args.counters == nullptr) continue;  // rvq_apply_kernel merges the splits
        // Split fixup: publish this split's partials, count the arrival; the
        // CTA completing the row block merges all splits (lowest distance,
        // then lowest index) and carries on as if it had owned every code.
        // (bounded mbarrier handshakes among the 4 argmin warps, so an abort cannot strand a warp)
        __threadfence();
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.fix_arrive);
        if (warp == 2) {
          int fine = 1;
          if (lane == 0) {
            fine = mbar_wait(&S.fix_arrive, fix_ph, abort_flag) ? 1 : 0;
            if (fine) {
              const int prev = atomicAdd(args.counters + rb, 1);
              const int last = prev == args.splits - 1;
              if (last) atomicExch(args.counters + rb, 0);  // ready for the next launch
              *reinterpret_cast<volatile int*>(&S.fix_last) = last;
              mbar_arrive(&S.fix_done);
            }
          }
          if (!__shfl_sync(0xffffffffu, fine, 0)) {
            ok = false;
            break;
          }
        }
        if (!mbar_wait(&S.fix_done, fix_ph, abort_flag)) {
          ok = false;
          break;
        }
        fix_ph ^= 1u;
        if (!*reinterpret_cast<volatile int*>(&S.fix_last)) continue;
        __threadfence();
        if (row < args.N) {
          float bd = INFINITY;
          int bi = INT_MAX;
          for (int s2i = 0; s2i < args.splits; ++s2i) {
            // L2 reads: the other splits were written by other SMs
            const int2 pv = __ldcg(reinterpret_cast<const int2*>(args.part + static_cast<size_t>(s2i) * args.N + row));
            const float d = __int_as_float(pv.x);
            if (d < bd || (d == bd && pv.y < bi)) {
              bd = d;
              bi = pv.y;
            }
          }
          if (bi == INT_MAX) bi = __ldcg(reinterpret_cast<const int2*>(args.part + row)).y;  // all NaN/inf
          bidx = bi;
          args.codes[row] = bidx;
        }
      }
      if (args.fuse) {
        const uint32_t ub = uit & 1u, up = (uit >> 1) & 1u;
        if (!mbar_wait(&S.upd_empty[ub], up ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        S.codes_s[ub][q * 32 + lane] = row < args.N ? bidx : -1;
        if (lane == 0) S.upd_rb[ub] = rb;
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.upd_full[ub]);
        ++uit;
      }
    }
    if (ok && args.fuse) {
      // end of work: tell the update warps
      const uint32_t ub = uit & 1u, up = (uit >> 1) & 1u;
      if (mbar_wait(&S.upd_empty[ub], up ^ 1u, abort_flag)) {
        if (lane == 0) S.upd_rb[ub] = -1;
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.upd_full[ub]);
      } else {
        ok = false;
      }
    }
    if (!ok) abort_all();
  } else if (args.fuse) {
    // ------------------------------------------------- residual update
    // Warp uw updates rows uw*16.. of each finished row block: one row at a
    // time, lanes striding the row in 16-byte (f32) / 8-byte (bf16) pieces.
    const int uw = warp - 6;
    uint32_t uit = 0;
    bool ok = true;
    for (;;) {
      const uint32_t ub = uit & 1u, up = (uit >> 1) & 1u;
      if (!mbar_wait(&S.upd_full[ub], up, abort_flag)) {
        ok = false;
        break;
      }
      const int rb = *reinterpret_cast<volatile int*>(&S.upd_rb[ub]);
      if (rb < 0) break;  // the epilogue has no more row blocks
      for (int r = 0; r < UPD_ROWS; ++r) {
        const int code = S.codes_s[ub][uw * UPD_ROWS + r];
        if (code < 0) continue;
        if (code >= args.K) {
          if (lane == 0) atomicOr(args.err, kErrBadIndex);
          continue;
        }
        const size_t ro = static_cast<size_t>(rb * BM + uw * UPD_ROWS + r) * args.D;
        const uint16_t* e = args.codebook + static_cast<size_t>(code) * args.D;
        // 1024 columns per batch: every load of the batch is issued before the
        // first store (the stores may alias later loads as far as the compiler
        // knows, so an interleaved loop keeps one load in flight per lane)
        for (int d0 = 0; d0 < args.D; d0 += 1024) {
          float4 x[8];
          uint2 ev[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int d = d0 + lane * 4 + j * 128;
            if (d < args.D) {
              if (args.src_bf16 != nullptr) {
                const uint2 sv = *reinterpret_cast<const uint2*>(args.src_bf16 + ro + d);
                x[j] = make_float4(bf16lo(sv.x), bf16hi(sv.x), bf16lo(sv.y), bf16hi(sv.y));
              } else {
                x[j] = *reinterpret_cast<const float4*>(args.resid + ro + d);
              }
              ev[j] = __ldg(reinterpret_cast<const uint2*>(e + d));
            }
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int d = d0 + lane * 4 + j * 128;
            if (d < args.D) {
              float4 v = x[j];
              v.x -= bf16lo(ev[j].x);
              v.y -= bf16hi(ev[j].x);
              v.z -= bf16lo(ev[j].y);
              v.w -= bf16hi(ev[j].y);
              *reinterpret_cast<float4*>(args.resid + ro + d) = v;
              if (args.shadow != nullptr)
                *reinterpret_cast<uint2*>(args.shadow + ro + d) =
                    make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.upd_empty[ub]);
      ++uit;
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
      tmem_dealloc_pair(tmem, TMEM_COLS);
    else
      tmem_dealloc(tmem, TMEM_COLS);
  }
}

// -------------------------------------------------------------- apply
// One warp per row: final code (reducing split partials lexicographically by
// (distance, index)), then the f32 residual update and its bf16 shadow.
struct ApplyArgs {
  const RvqPartial* part;
  int splits;
  int32_t* codes;
  const uint16_t* src_bf16;
  float* resid;
  uint16_t* shadow;
  const uint16_t* codebook;
  int* err;
  int N, D, K;
  int update;
  float* gap;            // [N] relative top-2 gap, or null
  const float* a2;       // [N] ||bf16(r)||^2 (with gap)
  const float* part_d2;  // [splits, N] second-smallest distance per split (with gap)
};

__global__ void __launch_bounds__(256) rvq_apply_kernel(const ApplyArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= a.N) return;
  int code;
  if (a.splits > 1) {
    float bd = INFINITY;
    int bi = INT_MAX;
    for (int s = lane; s < a.splits; s += 32) {
      const RvqPartial p = a.part[static_cast<size_t>(s) * a.N + row];
      if (p.d < bd || (p.d == bd && p.idx < bi)) {
        bd = p.d;
        bi = p.idx;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float od = __shfl_xor_sync(0xffffffffu, bd, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (od < bd || (od == bd && oi < bi)) {
        bd = od;
        bi = oi;
      }
    }
    code = bi;
    if (code == INT_MAX) code = a.part[row].idx;  // every distance was NaN/inf
    if (lane == 0) a.codes[row] = code;
    if (a.gap != nullptr) {
      // the two smallest distances over all splits: merge (smallest, second) pairs
      float s1 = INFINITY, s2 = INFINITY;
      for (int s = lane; s < a.splits; s += 32) {
        const float d1 = a.part[static_cast<size_t>(s) * a.N + row].d;
        const float d2 = a.part_d2[static_cast<size_t>(s) * a.N + row];
        s2 = fminf(fmaxf(s1, d1), fminf(s2, d2));
        s1 = fminf(s1, d1);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float o1 = __shfl_xor_sync(0xffffffffu, s1, o);
        const float o2 = __shfl_xor_sync(0xffffffffu, s2, o);
        s2 = fminf(fmaxf(s1, o1), fminf(s2, o2));
        s1 = fminf(s1, o1);
      }
      if (lane == 0) a.gap[row] = rel_gap(s1, s2, a.a2[row]);
    }
  } else {
    code = a.codes[row];
  }
  if (!a.update) return;
  if (code < 0 || code >= a.K) {
    if (lane == 0) atomicOr(a.err, kErrBadIndex);
    return;
  }
  const size_t ro = static_cast<size_t>(row) * a.D;
  const uint16_t* e = a.codebook + static_cast<size_t>(code) * a.D;
  // 1024 columns per batch, every load of the batch issued before the first
  // store: the stores may alias later loads as far as the compiler knows, so
  // a plain loop keeps one residual and one codeword load in flight per lane
  for (int d0 = 0; d0 < a.D; d0 += 1024) {
    float4 x[8];
    uint2 ev[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int d = d0 + lane * 4 + j * 128;
      if (d < a.D) {
        if (a.src_bf16 != nullptr) {
          const uint2 sv = *reinterpret_cast<const uint2*>(a.src_bf16 + ro + d);
          x[j] = make_float4(bf16lo(sv.x), bf16hi(sv.x), bf16lo(sv.y), bf16hi(sv.y));
        } else {
          x[j] = *reinterpret_cast<const float4*>(a.resid + ro + d);
        }
        ev[j] = __ldg(reinterpret_cast<const uint2*>(e + d));
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int d = d0 + lane * 4 + j * 128;
      if (d < a.D) {
        float4 r = x[j];
        r.x -= bf16lo(ev[j].x);
        r.y -= bf16hi(ev[j].x);
        r.z -= bf16lo(ev[j].y);
        r.w -= bf16hi(ev[j].y);
        *reinterpret_cast<float4*>(a.resid + ro + d) = r;
        if (a.shadow != nullptr)
          *reinterpret_cast<uint2*>(a.shadow + ro + d) = make_uint2(pack_bf16x2(r.x, r.y), pack_bf16x2(r.z, r.w));
      }
    }
  }
}

// ---------------------------------------------------------- sqnorm (R1)
// One warp per code; squares of bf16 values are exact in f64 and their sum is
// exact for any realistic D, so the f32 result does not depend on order.
__global__ void __launch_bounds__(256) code_sqnorm_kernel(const uint16_t* __restrict__ cb, float* __restrict__ out,
                                                          int K, int D) {
  pdl_wait();
  pdl_launch_dependents();
  const int k = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (k >= K) return;
  const uint16_t* e = cb + static_cast<size_t>(k) * D;
  double s = 0.0;
  for (int d = lane * 2; d < D; d += 64) {
    const uint32_t p = *reinterpret_cast<const uint32_t*>(e + d);
    const double lo = bf16lo(p), hi = bf16hi(p);
    s += lo * lo + hi * hi;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) out[k] = static_cast<float>(s);
}

// ------------------------------------------------------------ decode (R5)
// One warp per row: recon[n] = sum_l e_l[codes[l,n]] in f32, level order.
// The row's codes are checked first (lane i holds level l32 + i of each
// 32-level group), so a row with an out-of-range code is left unwritten.
// Each lane then covers 8 columns (16 bytes) of a 256-column chunk, and the
// codeword pieces of up to 8 levels are all loaded before the first add: a
// warp keeps 8 gathers in flight instead of one dependent code-then-codeword
// pair per level.
__global__ void __launch_bounds__(256) rvq_decode_kernel(const int32_t* __restrict__ codes,
                                                         const uint16_t* __restrict__ cbs, int L,
                                                         uint16_t* __restrict__ out_bf16,
                                                         float* __restrict__ out_f32, int N, int D, int K,
                                                         int* err) {
  pdl_wait();
  pdl_launch_dependents();
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= N) return;  // whole warps leave together
  bool bad = false;
  for (int l32 = 0; l32 < L; l32 += 32) {
    if (l32 + lane < L) {
      const int c = __ldg(codes + static_cast<size_t>(l32 + lane) * N + row);
      bad |= (c < 0 || c >= K);
    }
  }
  if (__any_sync(0xffffffffu, bad)) {
    if (lane == 0) atomicOr(err, kErrBadIndex);
    return;
  }
  const size_t ro = static_cast<size_t>(row) * D;
  for (int d0 = 0; d0 < D; d0 += 256) {
    const int d = d0 + lane * 8;
    const bool act = d < D;
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    for (int l32 = 0; l32 < L; l32 += 32) {
      const int mine = (l32 + lane < L) ? __ldg(codes + static_cast<size_t>(l32 + lane) * N + row) : 0;
      const int lend = min(L - l32, 32);
      for (int g = 0; g < lend; g += 8) {
        uint4 ev[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int c = __shfl_sync(0xffffffffu, mine, (g + j) & 31);
          if (g + j < lend && act)
            ev[j] = __ldg(reinterpret_cast<const uint4*>(
                cbs + (static_cast<size_t>(l32 + g + j) * K + c) * D + d));
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (g + j < lend && act) {
            acc[0] += bf16lo(ev[j].x);
            acc[1] += bf16hi(ev[j].x);
            acc[2] += bf16lo(ev[j].y);
            acc[3] += bf16hi(ev[j].y);
            acc[4] += bf16lo(ev[j].z);
            acc[5] += bf16hi(ev[j].z);
            acc[6] += bf16lo(ev[j].w);
            acc[7] += bf16hi(ev[j].w);
          }
        }
      }
    }
    if (act) {
      if (out_bf16 != nullptr)
        *reinterpret_cast<uint4*>(out_bf16 + ro + d) =
            make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]), pack_bf16x2(acc[4], acc[5]),
                       pack_bf16x2(acc[6], acc[7]));
      if (out_f32 != nullptr) {
        *reinterpret_cast<float4*>(out_f32 + ro + d) = make_float4(acc[0], acc[1], acc[2], acc[3]);
        *reinterpret_cast<float4*>(out_f32 + ro + d + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
      }
    }
  }
}

// -------------------------------------------------------------- pool (R4)
// y[b,j,:] = (sum_{i<f} x[b,j*f+i,:]) / f, increasing i, f32. One thread per
// 4 channels of one output row.
__global__ void __launch_bounds__(256) pool_avg_kernel(const float* __restrict__ x, float* __restrict__ y,
                                                       uint16_t* __restrict__ y_bf16, long long rows_out, int D,
                                                       int f) {
  pdl_wait();
  pdl_launch_dependents();
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int d4 = D / 4;
  if (idx >= rows_out * d4) return;
  const long long orow = idx / d4;
  const int d = static_cast<int>(idx - orow * d4) * 4;
  const float* src = x + orow * f * D + d;
  float4 s = *reinterpret_cast<const float4*>(src);
  for (int i = 1; i < f; ++i) {
    const float4 v = *reinterpret_cast<const float4*>(src + static_cast<size_t>(i) * D);
    s.x += v.x;
    s.y += v.y;
    s.z += v.z;
    s.w += v.w;
  }
  const float inv = static_cast<float>(f);
  s.x /= inv;
  s.y /= inv;
  s.z /= inv;
  s.w /= inv;
  *reinterpret_cast<float4*>(y + orow * D + d) = s;
  if (y_bf16 != nullptr)
    *reinterpret_cast<uint2*>(y_bf16 + orow * D + d) = make_uint2(pack_bf16x2(s.x, s.y), pack_bf16x2(s.z, s.w));
}

// ------------------------------------------------- scale advance (R4+R6)
// One warp per pooled row p of scale s (factor f): q = sum_l e_l[codes[l,p]]
// (f32, level order) is stored to q_out[p]; when a next scale exists (factor
// g dividing f) the f full-resolution rows get r -= q and are pooled on the
// fly into u_next (same summation order as pool_avg_kernel) with its bf16
// shadow. The residual is updated only when a next scale needs it.
__global__ void __launch_bounds__(256) scale_advance_kernel(const int32_t* __restrict__ codes,
                                                            const uint16_t* __restrict__ cbs, int L,
                                                            float* __restrict__ resid, float* __restrict__ q_out,
                                                            float* __restrict__ u_next,
                                                            uint16_t* __restrict__ u_next_bf16, long long rows_pooled,
                                                            int D, int K, int f, int g, int update_r, int* err) {
  pdl_wait();
  pdl_launch_dependents();
  // one warp per (pooled row, 128-channel chunk)
  const int nch = (D + 127) / 128;
  const long long wg = static_cast<long long>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const long long p = wg / nch;
  const int ch = static_cast<int>(wg - p * nch);
  const int lane = threadIdx.x & 31;
  if (p >= rows_pooled) return;
  // Levels in groups of eight: lanes 0-7 read the group's codes (checked
  // before any use), then the eight codeword gathers are issued together and
  // summed in level order.
  const int d = ch * 128 + lane * 4;
  const bool act = d < D;
  float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int l0 = 0; l0 < L; l0 += 8) {
    const int nl = min(8, L - l0);
    const int mc = lane < nl ? __ldg(codes + static_cast<size_t>(l0 + lane) * rows_pooled + p) : 0;
    if (__any_sync(0xffffffffu, lane < nl && (mc < 0 || mc >= K))) {
      if (lane == 0 && ch == 0) atomicOr(err, kErrBadIndex);
      return;
    }
    uint2 ev[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = __shfl_sync(0xffffffffu, mc, j);
      ev[j] = make_uint2(0u, 0u);
      if (j < nl && act)
        ev[j] = __ldg(reinterpret_cast<const uint2*>(cbs + (static_cast<size_t>(l0 + j) * K + c) * D + d));
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j < nl) {
        q.x += bf16lo(ev[j].x);
        q.y += bf16hi(ev[j].x);
        q.z += bf16lo(ev[j].y);
        q.w += bf16hi(ev[j].y);
      }
    }
  }
  if (!act) return;
  *reinterpret_cast<float4*>(q_out + static_cast<size_t>(p) * D + d) = q;
  if (!update_r) return;
  float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
  // The rows are read in batches of kBatch before any of them is written back:
  // loads and stores share one pointer with a run-time row stride, so without
  // the batching each load would wait for the previous row's store.
  constexpr int kBatch = 4;
  for (int i0 = 0; i0 < f; i0 += kBatch) {
    float4 r[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; ++j)
      if (i0 + j < f)
        r[j] = *reinterpret_cast<const float4*>(resid + (static_cast<size_t>(p) * f + i0 + j) * D + d);
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int i = i0 + j;
      if (i >= f) break;
      const size_t row = static_cast<size_t>(p) * f + i;
      r[j].x -= q.x;
      r[j].y -= q.y;
      r[j].z -= q.z;
      r[j].w -= q.w;
      *reinterpret_cast<float4*>(resid + row * D + d) = r[j];
      if (g <= 0) continue;
      if (i % g == 0) {
        sum = r[j];
      } else {
        sum.x += r[j].x;
        sum.y += r[j].y;
        sum.z += r[j].z;
        sum.w += r[j].w;
      }
      if (i % g == g - 1) {
        const float gf = static_cast<float>(g);
        const float4 u = make_float4(sum.x / gf, sum.y / gf, sum.z / gf, sum.w / gf);
        const size_t urow = row / g;
        *reinterpret_cast<float4*>(u_next + urow * D + d) = u;
        *reinterpret_cast<uint2*>(u_next_bf16 + urow * D + d) =
            make_uint2(pack_bf16x2(u.x, u.y), pack_bf16x2(u.z, u.w));
      }
    }
  }
}

// recon[t] = bf16(sum_s q_s[t / f_s]) over scales in order (f32), one thread per 4 channels
struct ReconArgs {
  const float* q[16];
  int f[16];
  int S;
};
__global__ void __launch_bounds__(256) multiscale_recon_kernel(const ReconArgs a, uint16_t* __restrict__ out,
                                                               long long rows, int D) {
  pdl_wait();
  pdl_launch_dependents();
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int d4 = D / 4;
  if (idx >= rows * d4) return;
  const long long t = idx / d4;
  const int d = static_cast<int>(idx - t * d4) * 4;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s = 0; s < a.S; ++s) {
    const float4 q = *reinterpret_cast<const float4*>(a.q[s] + (t / a.f[s]) * D + d);
    acc.x += q.x;
    acc.y += q.y;
    acc.z += q.z;
    acc.w += q.w;
  }
  *reinterpret_cast<uint2*>(out + t * D + d) = make_uint2(pack_bf16x2(acc.x, acc.y), pack_bf16x2(acc.z, acc.w));
}

// ------------------------------------------------------------ casts (L7)
__global__ void __launch_bounds__(256) f32_to_bf16_kernel(const float* __restrict__ x, uint16_t* __restrict__ y,
                                                          long long n) {
  pdl_wait();
  pdl_launch_dependents();
  const long long i = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
  if (i + 3 < n) {
    const float4 v = *reinterpret_cast<const float4*>(x + i);
    *reinterpret_cast<uint2*>(y + i) = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
  } else {
    for (long long j = i; j < n; ++j) y[j] = f32_to_bf16(x[j]);
  }
}

__global__ void __launch_bounds__(256) bf16_to_f32_kernel(const uint16_t* __restrict__ x, float* __restrict__ y,
                                                          long long n) {
  pdl_wait();
  pdl_launch_dependents();
  const long long i = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
  if (i + 3 < n) {
    const uint2 v = *reinterpret_cast<const uint2*>(x + i);
    *reinterpret_cast<float4*>(y + i) = make_float4(bf16lo(v.x), bf16hi(v.x), bf16lo(v.y), bf16hi(v.y));
  } else {
    for (long long j = i; j < n; ++j) y[j] = bf16_to_f32(x[j]);
  }
}

}  // namespace

// ================================================================== host

namespace {
// How many 2-CTA clusters of the pair kernel fit on this device at once
// (cluster placement can leave SMs idle); cached per device.
int max_active_pairs(int num_sms) {
  static std::atomic<int> cached[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return num_sms / 2;
  const int known = cached[dev].load(std::memory_order_relaxed);
  if (known > 0) return known;
  int n = 0;
  const size_t smem = argmin_smem_bytes<true>();
  if (cudaFuncSetAttribute(rvq_argmin_kernel<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) == cudaSuccess) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(2 * (num_sms / 2));
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, rvq_argmin_kernel<false, true>, &cfg) != cudaSuccess) n = 0;
  }
  cudaGetLastError();
  const int v = n > 0 ? std::min(n, num_sms / 2) : -1;
  cached[dev].store(v, std::memory_order_relaxed);  // every thread computes the same value
  return v;
}
}  // namespace

// Split count s minimising (waves x tiles per unit) for `blocks` row units
// on `slots` concurrent workers; fewer splits on ties, since every split adds
// a partial write and a reduction.
static void best_split(int blocks, int code_tiles, int slots, int& best_s, long long& best_cost) {
  best_cost = -1;
  best_s = 1;
  for (int s = 1; s <= code_tiles; ++s) {
    const int tps = ceil_div(code_tiles, s);
    const int s_eff = ceil_div(code_tiles, tps);
    if (s_eff != s) continue;
    const long long units = static_cast<long long>(blocks) * s;
    const long long waves = (units + slots - 1) / slots;
    const long long cost = waves * tps;
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best_s = s;
    }
  }
}

RvqPlan rvq_plan(int num_sms, int64_t N, int64_t K, bool allow_pair) {
  RvqPlan p{};
  p.row_blocks = ceil_div(N, BM);
  p.code_tiles = ceil_div(K, BN);
  // one-CTA units: (128-row block, code range) on every SM; with enough row
  // blocks for every SM there is no code split, so the residual update can
  // run inside the distance kernel
  int s1 = 1;
  long long cost1 = 0;
  if (p.row_blocks >= num_sms)
    cost1 = static_cast<long long>(ceil_div(p.row_blocks, num_sms)) * p.code_tiles;
  else
    best_split(p.row_blocks, p.code_tiles, num_sms, s1, cost1);
  p.splits = s1;
  p.tiles_per_split = ceil_div(p.code_tiles, s1);
  p.n_units = p.row_blocks * s1;
  p.grid = p.n_units < num_sms ? p.n_units : num_sms;
  p.partial_bytes = s1 > 1 ? static_cast<size_t>(s1) * N * sizeof(RvqPartial) : 0;
  if (allow_pair) {
    // CTA pairs: one MMA over 256 rows, each CTA loading half of every code
    // tile, so a pair's tile step costs a one-CTA step in time with a third
    // less operand traffic per SM and deeper staging. Used whenever its step
    // count (waves x tiles per unit over the pairs) is no larger.
    const int pairs = max_active_pairs(num_sms);
    const int units = ceil_div(N, 2 * BM);
    if (pairs > 0) {
      int s2 = 1;
      long long cost2 = 0;
      if (units >= pairs)
        cost2 = static_cast<long long>(ceil_div(units, pairs)) * p.code_tiles;
      else
        best_split(units, p.code_tiles, pairs, s2, cost2);
      if (cost2 <= cost1) {
        p.pair = 1;
        p.splits = s2;
        p.tiles_per_split = ceil_div(p.code_tiles, s2);
        p.n_units = units * s2;
        p.grid = 2 * (p.n_units < pairs ? p.n_units : pairs);  // every pair gets at least one unit
        p.partial_bytes = s2 > 1 ? static_cast<size_t>(s2) * N * sizeof(RvqPartial) : 0;
      }
    }
  }
  return p;
}

cudaError_t launch_rvq_argmin(const RvqPlan& plan, const CUtensorMap& tmA, const CUtensorMap& tmB,
                              const float* sqnorm, int32_t* codes, RvqPartial* part, int* err, int64_t N,
                              int64_t D, int64_t K, cudaStream_t stream, const RvqFusedUpdate* fu,
                              const RvqTop2* top2, const float* mul_dev, int* counters) {
  if (plan.pair && top2 != nullptr) return cudaErrorInvalidValue;
  // the shared-memory opt-in is per device and per instantiation: remember which devices have it
  static DeviceFlags attr_set[3];
  const int gi = plan.pair ? 2 : (top2 != nullptr ? 1 : 0);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (!attr_set[gi].test(dev)) {
    if (gi == 2)
      e = cudaFuncSetAttribute(rvq_argmin_kernel<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(argmin_smem_bytes<true>()));
    else if (gi == 1)
      e = cudaFuncSetAttribute(rvq_argmin_kernel<true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(argmin_smem_bytes<false>()));
    else
      e = cudaFuncSetAttribute(rvq_argmin_kernel<false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(argmin_smem_bytes<false>()));
    if (e != cudaSuccess) return e;
    attr_set[gi].set(dev);
  }
  ArgminArgs a{};
  a.csq = sqnorm;
  a.codes = codes;
  a.part = part;
  a.err = err;
  a.N = static_cast<int>(N);
  a.D = static_cast<int>(D);
  a.K = static_cast<int>(K);
  a.splits = plan.splits;
  a.tiles_per_split = plan.tiles_per_split;
  a.code_tiles = plan.code_tiles;
  a.n_units = plan.n_units;
  // the split fixup needs counters, does not carry the top-2 gap, and writes
  // codes only (an update after a split plan is rvq_apply_kernel's)
  a.counters = (plan.splits > 1 && top2 == nullptr && fu == nullptr) ? counters : nullptr;
  a.fuse = (fu != nullptr && plan.splits == 1) ? 1 : 0;
  a.resid = fu ? fu->resid : nullptr;
  a.src_bf16 = fu ? fu->src_bf16 : nullptr;
  a.shadow = fu ? fu->shadow : nullptr;
  a.codebook = fu ? fu->codebook : nullptr;
  a.mul_dev = mul_dev;
  if (plan.pair)
    return launch_pdl(rvq_argmin_kernel<false, true>, dim3(plan.grid), dim3(THREADS), argmin_smem_bytes<true>(),
                      stream, 2, tmA, tmB, a);
  if (top2 != nullptr) {
    a.gap = top2->gap;
    a.a2 = top2->a2;
    a.part_d2 = top2->part_d2;
    return launch_pdl(rvq_argmin_kernel<true, false>, dim3(plan.grid), dim3(THREADS), argmin_smem_bytes<false>(),
                      stream, 1, tmA, tmB, a);
  }
  return launch_pdl(rvq_argmin_kernel<false, false>, dim3(plan.grid), dim3(THREADS), argmin_smem_bytes<false>(), stream,
                    1, tmA, tmB, a);
}

cudaError_t launch_rvq_apply(const RvqPlan& plan, const RvqPartial* part, int32_t* codes, const uint16_t* src_bf16,
                             float* resid, uint16_t* shadow, const uint16_t* codebook, int* err, int64_t N,
                             int64_t D, int64_t K, bool update, cudaStream_t stream, const RvqTop2* top2) {
  if (plan.splits == 1 && !update) return cudaSuccess;
  ApplyArgs a{};
  if (top2 != nullptr && plan.splits > 1) {
    a.gap = top2->gap;
    a.a2 = top2->a2;
    a.part_d2 = top2->part_d2;
  }
  a.part = part;
  a.splits = plan.splits;
  a.codes = codes;
  a.src_bf16 = src_bf16;
  a.resid = resid;
  a.shadow = shadow;
  a.codebook = codebook;
  a.err = err;
  a.N = static_cast<int>(N);
  a.D = static_cast<int>(D);
  a.K = static_cast<int>(K);
  a.update = update ? 1 : 0;
  return launch_pdl(rvq_apply_kernel, dim3(ceil_div(N, 8)), dim3(256), 0, stream, 1, a);
}

cudaError_t launch_code_sqnorm(const uint16_t* codebook, float* sqnorm, int64_t K, int64_t D, cudaStream_t stream) {
  return launch_pdl(code_sqnorm_kernel, dim3(ceil_div(K, 8)), dim3(256), 0, stream, 1, codebook, sqnorm,
                    static_cast<int>(K), static_cast<int>(D));
}

cudaError_t launch_rvq_decode(const int32_t* codes, const uint16_t* codebooks, int L, uint16_t* recon_bf16,
                              float* recon_f32, int64_t N, int64_t D, int64_t K, int* err, cudaStream_t stream) {
  return launch_pdl(rvq_decode_kernel, dim3(ceil_div(N, 8)), dim3(256), 0, stream, 1, codes, codebooks, L, recon_bf16,
                    recon_f32, static_cast<int>(N), static_cast<int>(D), static_cast<int>(K), err);
}

cudaError_t launch_pool_avg(const float* x, float* y, uint16_t* y_bf16, int64_t B, int64_t T, int64_t D, int f,
                            cudaStream_t stream) {
  const long long rows_out = B * (T / f);
  const long long threads = rows_out * (D / 4);
  return launch_pdl(pool_avg_kernel, dim3(static_cast<unsigned>((threads + 255) / 256)), dim3(256), 0, stream, 1, x, y,
                    y_bf16, rows_out, static_cast<int>(D), f);
}

cudaError_t launch_scale_advance(const int32_t* codes, const uint16_t* codebooks, int L, float* resid, float* q_out,
                                 float* u_next, uint16_t* u_next_bf16, int64_t rows_pooled, int64_t D, int64_t K, int f,
                                 int g, bool update_r, int* err, cudaStream_t stream) {
  const long long warps = rows_pooled * ((D + 127) / 128);
  return launch_pdl(scale_advance_kernel, dim3(static_cast<unsigned>((warps + 7) / 8)), dim3(256), 0, stream, 1, codes,
                    codebooks, L, resid, q_out, u_next, u_next_bf16, static_cast<long long>(rows_pooled),
                    static_cast<int>(D), static_cast<int>(K), f, g, update_r ? 1 : 0, err);
}

cudaError_t launch_multiscale_recon(const float* const* q, const int* f, int S, uint16_t* out, int64_t rows, int64_t D,
                                    cudaStream_t stream) {
  ReconArgs a{};
  a.S = S;
  for (int s = 0; s < S; ++s) {
    a.q[s] = q[s];
    a.f[s] = f[s];
  }
  const long long threads = rows * (D / 4);
  return launch_pdl(multiscale_recon_kernel, dim3(static_cast<unsigned>((threads + 255) / 256)), dim3(256), 0, stream, 1,
                    a, out, static_cast<long long>(rows), static_cast<int>(D));
}

cudaError_t launch_f32_to_bf16(const float* x, uint16_t* y, int64_t n, cudaStream_t stream) {
  const long long threads = (n + 3) / 4;
  if (threads == 0) return cudaSuccess;
  return launch_pdl(f32_to_bf16_kernel, dim3(static_cast<unsigned>((threads + 255) / 256)), dim3(256), 0, stream, 1, x,
                    y, static_cast<long long>(n));
}

cudaError_t launch_bf16_to_f32(const uint16_t* x, float* y, int64_t n, cudaStream_t stream) {
  const long long threads = (n + 3) / 4;
  if (threads == 0) return cudaSuccess;
  return launch_pdl(bf16_to_f32_kernel, dim3(static_cast<unsigned>((threads + 255) / 256)), dim3(256), 0, stream, 1, x,
                    y, static_cast<long long>(n));
}

}  // namespace ncm
