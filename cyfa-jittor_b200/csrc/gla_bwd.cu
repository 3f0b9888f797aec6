// Backward of the chunked CyFA op on tcgen05.
//
// For one ScalarGatedLA pass with tile states S_j (forward history) and state
// adjoints H_{j+1} (reverse scan, state_scan_kernel<true>), and the masked tile
// score matrices
//   A_ts  = [s<=t] scale 2^{G_t-G_s} (q_t . k_s)
//   B'_ts = [s<=t] scale 2^{G_t-G_s} (dO_t . v_s)
// the adjoints are
//   dq_t = sum_s B'_ts k_s + scale 2^{G_t} dO_t S_j^T
//   dk_s = sum_t B'_ts q_t + 2^{G_L-G_s} v_s H_{j+1}^T
//   dv_s = sum_t A_ts dO_t + 2^{G_L-G_s} k_s H_{j+1}
//   dG_t = q_t . dq_t - k_t . dk_t + [t = L] <S_{j+1}, H_{j+1}>   (natural-log units)
// (the reference's scalar_grad, cyclic_flow_attention/ops/chunk_bwd.py:1015-1041,
// with its "force" and "boundary" gate terms at :203-235,247-272).
//
// tile_scores_kernel : A and B' of a tile (two 128x128 UMMAs + masked epilogue).
// dual_gemm_kernel   : out = X1 Y1 + r_t (X2 Y2) for one tile, the shape shared by
//                      dq, dk and dv of both passes; X1 is A or B' (or its
//                      transpose), r_t the per-row decay factor, plus an optional
//                      per-row dot product folded into dG.
// readout_bwd_kernel : adjoint of the softmax slot readout (ops/chunk_readout.py:401-621):
//                      dcoeff = U(lam) dw, dp = dcoeff Table^T, dl = p o (dp - <p,dp>),
//                      dz = dl Table, draw = U(-lam) dz, dlam from the rotations,
//                      and the tile's partial dTable = p^T dcoeff + dl^T z.
#include "cyfa_common.cuh"
#include "phase.cuh"

namespace cyfa {

// ============================================================ tile scores
struct ScoresParams {
  int BH, H, TP, NT;
  int DK, DV;
  int do_mode, v_mode;
  const float* G;
  float scale;
  __nv_bfloat16* A;   // [BH*NT*128, 128]
  __nv_bfloat16* Bp;  // [BH*NT*128, 128]
};

constexpr int kScoresStage = 32768;  // one 64-wide k-block of both operands
constexpr int kScoresStages = 6;
constexpr int kScoresBufs = 4;       // TMEM accumulators of 128 columns
constexpr int kScoresSmem = kScoresStages * kScoresStage + 8 * 2048 + 1024;
constexpr int kScoresThreads = 320;

// Persistent and warp-specialised like dual_gemm_kernel.  A unit is one score
// matrix of one tile: units 0..ntiles-1 are A (q.k over DK), the next ntiles B'
// (dO.v over DV), so every CTA gets a share of both kinds.  The unit's GEMM
// streams 64-wide k-blocks (the q and k blocks, or the dO and v blocks, 32 KiB)
// through a ring of stages:
//   warp 8, lane 0: TMA loads;  warp 9, lane 0: the UMMAs into one of four TMEM
//   accumulators;  warps 0-7: the masked, decayed epilogue (warp w: TMEM lane
//   quadrant w & 3 = token rows, column half w >> 2) and the bf16 stores.
__global__ void __launch_bounds__(kScoresThreads, 1)
    tile_scores_kernel(const __grid_constant__ CUtensorMap map_q,
                       const __grid_constant__ CUtensorMap map_k,
                       const __grid_constant__ CUtensorMap map_do,
                       const __grid_constant__ CUtensorMap map_v, ScoresParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  __shared__ __align__(8) uint64_t full[kScoresStages], empty[kScoresStages];
  __shared__ __align__(8) uint64_t acc_full[kScoresBufs], acc_empty[kScoresBufs];
  __shared__ uint32_t tmem_base;
  __shared__ int s_abort;
  volatile int* abort_flag = &s_abort;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ntiles = p.BH * p.NT, nunits = 2 * ntiles;
  if (tid == 0) {
    for (int i = 0; i < kScoresStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < kScoresBufs; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 8);
    }
    s_abort = 0;
    mbar_fence_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base, 128 * kScoresBufs);
    tmem_relinquish();  // one allocation per CTA: let co-resident CTAs allocate
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();
  pdl_trigger();
  const uint32_t tmem = tmem_base;

  if (warp == 8) {
    // ------------------------------------------------ producer
    if (lane == 0) {
      int it = 0;
      for (int u = blockIdx.x; u < nunits && !*abort_flag; u += gridDim.x) {
        const bool bp = u >= ntiles;
        const int tile = bp ? u - ntiles : u, bh = tile / p.NT, j = tile % p.NT;
        const int nkb = (bp ? p.DV : p.DK) / 64;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % kScoresStages;
          if (it >= kScoresStages &&
              !mbar_wait(&empty[s], ((it / kScoresStages) - 1) & 1)) {
            *abort_flag = 1;
            break;
          }
          uint8_t* xb = smem + s * kScoresStage;
          mbar_expect_tx(&full[s], kScoresStage);
          if (bp) {
            load_token_tile(xb, &map_do, p.do_mode, bh, p.H, p.TP, j, 64 * kb, 64, &full[s]);
            load_token_tile(xb + 16384, &map_v, p.v_mode, bh, p.H, p.TP, j, 64 * kb, 64, &full[s]);
          } else {
            load_token_tile(xb, &map_q, kRows2D, bh, p.H, p.TP, j, 64 * kb, 64, &full[s]);
            load_token_tile(xb + 16384, &map_k, kRows2D, bh, p.H, p.TP, j, 64 * kb, 64, &full[s]);
          }
        }
      }
      // every issued copy lands before shared memory goes away
      for (int i = it > kScoresStages ? it - kScoresStages : 0; i < it; ++i)
        mbar_wait(&full[i % kScoresStages], (i / kScoresStages) & 1);
    }
  } else if (warp == 9) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = make_idesc(128, 128, 0, 0);
      int it = 0, tl = 0;
      uint64_t* last_bar = nullptr;
      uint32_t last_par = 0;
      for (int u = blockIdx.x; u < nunits && !*abort_flag; u += gridDim.x, ++tl) {
        const int nkb = (u >= ntiles ? p.DV : p.DK) / 64, b = tl % kScoresBufs;
        if (tl >= kScoresBufs && !mbar_wait(&acc_empty[b], ((tl / kScoresBufs) - 1) & 1)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % kScoresStages;
          if (!mbar_wait(&full[s], (it / kScoresStages) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t xb = smem_u32(smem + s * kScoresStage), yb = xb + 16384;
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            umma_bf16(tmem + 128 * b, kmaj_desc(xb, 128, ks), kmaj_desc(yb, 128, ks), idesc,
                      kb > 0 || ks > 0);
          umma_commit(&empty[s]);
          last_bar = &empty[s];
          last_par = (it / kScoresStages) & 1;
        }
        if (!ok) {
          *abort_flag = 1;
          break;
        }
        umma_commit(&acc_full[b]);
        last_bar = &acc_full[b];
        last_par = (tl / kScoresBufs) & 1;
      }
      if (last_bar) mbar_wait(last_bar, last_par);  // all issued MMAs are done
    }
  } else {
    // ------------------------------------------------ epilogue
    const int quad = warp & 3, half = warp >> 2;
    const int r = quad * 32 + lane;  // tile row = TMEM lane
    const uint32_t lane_tmem = tmem + ((quad * 32) << 16);
    const uint32_t scratch = smem_u32(smem) + kScoresStages * kScoresStage + warp * 2048;
    int tl = 0;
    for (int u = blockIdx.x; u < nunits; u += gridDim.x, ++tl) {
      const bool bp = u >= ntiles;
      const int tile = bp ? u - ntiles : u, bh = tile / p.NT, j = tile % p.NT;
      const int b = tl % kScoresBufs;
      // the gate cumsum of this row and of this warp's 64 columns (one per lane
      // and chunk, broadcast by shuffles), fetched before the MMAs are waited for
      const float* Gt = p.G + size_t(bh) * p.TP + j * 128;
      const float gt = Gt[r];
      const float gc0 = Gt[64 * half + lane], gc1 = Gt[64 * half + 32 + lane];
      const bool got = __all_sync(0xffffffffu, *abort_flag == 0 &&
                                                   mbar_wait(&acc_full[b], (tl / kScoresBufs) & 1));
      tc_fence_after();
      if (!got) {
        *abort_flag = 1;
        break;
      }
      __nv_bfloat16* out = (bp ? p.Bp : p.A) + (size_t(tile) * 128 + quad * 32) * 128;
#pragma unroll 1
      for (int cc = 0; cc < 2; ++cc) {
        const int c = 2 * half + cc;
        float a[32];
        if (c <= quad) {  // chunks above the diagonal block are all masked
          tmem_ld32(lane_tmem + 128 * b + 32 * c, a);
          const float gc = cc ? gc1 : gc0;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int s_ = 32 * c + i;
            const float gs = __shfl_sync(0xffffffffu, gc, i);
            a[i] *= s_ <= r ? p.scale * fast_exp2(gt - gs) : 0.f;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) a[i] = 0.f;
        }
        warp_store_block_bf16(scratch, a, out + 32 * c, 128, 0xffffffffu);
      }
      // hand the TMEM buffer back to the MMA issuer
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 128 * kScoresBufs);
  }
}

// ============================================================ dual GEMM
// One GEMM pair of a pass: out = X1 Y1 + r_t (X2 Y2) for every tile.
struct DualJob {
  int x1_mn;     // 0: X1 as stored ([t][s], K-major); 1: its transpose (MN-major)
  int y1_mode;   // token-row mode of Y1 [128 tok x N]
  int x2_mode;   // token-row mode of X2 [128 tok x KD]
  int y2_kmaj;   // 1: B2 = hist^T (N = hist rows); 0: B2 = hist (N = hist cols, KD rows)
  int N, KD;     // output columns (128 or 256), contraction of the second GEMM
  float scale;
  int fkind;     // row factor: 0 -> scale 2^{G_t}; 1 -> 2^{G_L - G_t}
  int out_mode;  // 0: fp32 [BH,TP,N]; 2: bf16 public [B,T,H,N]; 3: bf16 [BH,TP,N]
  void* out;
  long long out_stride;          // out_mode 2: elements between consecutive tokens
  const __nv_bfloat16* dot_src;  // optional [BH,TP,N] row-dot partner
  float dot_sign;
  float* dG;  // row-dot slots: column block nb writes dot_sign * <partner, out> to dG + nb*BH*TP
};

constexpr int kDualMaxJobs = 3;
constexpr int kDualMaxUnits = 6;  // per tile: sum over the jobs of N / 128

struct DualParams {
  int BH, H, TP, NT, T;
  const float* G;
  int units;  // units per tile
  int unit_job[kDualMaxUnits], unit_nb[kDualMaxUnits];
  DualJob job[kDualMaxJobs];
};

// Tensor maps of the jobs: X1, Y1, X2, Y2 each (box heights as the loads below use).
struct DualMaps {
  CUtensorMap x1[kDualMaxJobs], y1[kDualMaxJobs], x2[kDualMaxJobs], y2[kDualMaxJobs];
};

constexpr int kDualRing = 192 * 1024;                 // operand ring: 6 stages of 32 KiB
constexpr int kDualStage = 32768;
constexpr int kDualStages = kDualRing / kDualStage;
constexpr int kDualSmem = kDualRing + 8 * 2048 + 1024;  // + per-warp staging + alignment
constexpr int kDualThreads = 320;

// Persistent, warp-specialised, streaming over the contraction dimension.
// The work unit is one 128-column block of one job's output tile, and the units
// of a tile (every job of the pass, both column blocks of a 256-wide output)
// are consecutive, so the CTAs working side by side share the tile's operands
// through L2 and each operand is read from DRAM about once per pass.  A unit's
// two GEMMs are cut into 64-wide k-blocks (2 for X1 Y1, KD/64 for X2 Y2); a
// k-block stage holds one 128x64 block of the left operand and the matching
// 64x128 block of the right operand (32 KiB), and a ring of stages keeps the
// loads streaming across unit boundaries:
//   warp 8, lane 0 (producer): TMA loads into the ring;
//   warp 9, lane 0 (MMA issuer): the k-block UMMAs into the unit's TMEM buffer
//     (acc1 = X1 Y1 | acc2 = X2 Y2, 256 columns; two buffers), a commit per
//     stage frees it, a commit per unit hands the buffer over;
//   warps 0-7 (epilogue): warp w reads TMEM lane quadrant (w & 3) and column
//     half (w >> 2), forms out = acc1 + r_t acc2 (and the unit's share of the
//     row dot, written to its own dG slot).
// Operand boxes: X1 stored [t][s]; K-major X1 uses the 64-column panel of all
// 128 rows, MN-major X1 (its transpose) 64 rows x 128 columns.  Y1 (token rows)
// is read MN-major in 64-row blocks; Y2 (state history) K-major as a 64-column
// panel of 128 of its N rows, or MN-major in 64-row blocks.  Maps have the
// matching box heights (128, or 64 for the MN-major 64-row blocks).
__global__ void __launch_bounds__(kDualThreads, 1)
    dual_gemm_kernel(const __grid_constant__ DualMaps maps, const __grid_constant__ DualParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  __shared__ __align__(8) uint64_t full[kDualStages], empty[kDualStages];
  __shared__ __align__(8) uint64_t acc_full[2], acc_empty[2];
  __shared__ uint32_t tmem_base;
  __shared__ float dot_half[2][2][128];
  __shared__ int s_abort;
  volatile int* abort_flag = &s_abort;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nunits = p.BH * p.NT * p.units;
  if (tid == 0) {
    for (int i = 0; i < kDualStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 8);
    }
    s_abort = 0;
    mbar_fence_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base, 512);
    tmem_relinquish();  // one allocation per CTA: let co-resident CTAs allocate
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();
  pdl_trigger();
  const uint32_t tmem = tmem_base;

  if (warp == 8) {
    // ------------------------------------------------ producer
    if (lane == 0) {
      int it = 0;
      for (int u = blockIdx.x; u < nunits && !*abort_flag; u += gridDim.x) {
        const int tile = u / p.units, ui = u % p.units;
        const int ji = p.unit_job[ui], n0 = 128 * p.unit_nb[ui];
        const DualJob& jb = p.job[ji];
        const int bh = tile / p.NT, j = tile % p.NT, nkb = 2 + jb.KD / 64;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % kDualStages;
          if (it >= kDualStages && !mbar_wait(&empty[s], ((it / kDualStages) - 1) & 1)) {
            *abort_flag = 1;
            break;
          }
          uint8_t* xb = smem + s * kDualStage;
          uint8_t* yb = xb + 16384;
          mbar_expect_tx(&full[s], kDualStage);
          if (kb < 2) {
            if (jb.x1_mn) {
              tma_load_2d(xb, &maps.x1[ji], &full[s], 0, tile * 128 + 64 * kb);
              tma_load_2d(xb + 8192, &maps.x1[ji], &full[s], 64, tile * 128 + 64 * kb);
            } else {
              tma_load_2d(xb, &maps.x1[ji], &full[s], 64 * kb, tile * 128);
            }
            for (int c = 0; c < 2; ++c) {
              if (jb.y1_mode == kRows2D)
                tma_load_2d(yb + c * 8192, &maps.y1[ji], &full[s], n0 + 64 * c,
                            bh * p.TP + j * 128 + 64 * kb);
              else
                tma_load_4d(yb + c * 8192, &maps.y1[ji], &full[s], n0 + 64 * c, bh % p.H,
                            j * 128 + 64 * kb, bh / p.H);
            }
          } else {
            const int k2 = kb - 2;
            load_token_tile(xb, &maps.x2[ji], jb.x2_mode, bh, p.H, p.TP, j, 64 * k2, 64, &full[s]);
            if (jb.y2_kmaj) {
              tma_load_2d(yb, &maps.y2[ji], &full[s], 64 * k2, tile * jb.N + n0);
            } else {
              for (int c = 0; c < 2; ++c)
                tma_load_2d(yb + c * 8192, &maps.y2[ji], &full[s], n0 + 64 * c,
                            tile * jb.KD + 64 * k2);
            }
          }
        }
      }
      // every issued copy lands before shared memory goes away
      for (int i = it > kDualStages ? it - kDualStages : 0; i < it; ++i)
        mbar_wait(&full[i % kDualStages], (i / kDualStages) & 1);
    }
  } else if (warp == 9) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      int it = 0, tl = 0;
      uint64_t* last_bar = nullptr;
      uint32_t last_par = 0;
      for (int u = blockIdx.x; u < nunits && !*abort_flag; u += gridDim.x, ++tl) {
        const DualJob& jb = p.job[p.unit_job[u % p.units]];
        const uint32_t id1 = make_idesc(128, 128, jb.x1_mn, 1);
        const uint32_t id2 = make_idesc(128, 128, 0, jb.y2_kmaj ? 0 : 1);
        const int nkb = 2 + jb.KD / 64, b = tl & 1;
        if (tl >= 2 && !mbar_wait(&acc_empty[b], ((tl >> 1) - 1) & 1)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t acc1 = tmem + b * 256, acc2 = acc1 + 128;
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % kDualStages;
          if (!mbar_wait(&full[s], (it / kDualStages) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t xb = smem_u32(smem + s * kDualStage), yb = xb + 16384;
          if (kb < 2) {
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
              umma_bf16(acc1, jb.x1_mn ? mnmaj_desc(xb, 64, ks) : kmaj_desc(xb, 128, ks),
                        mnmaj_desc(yb, 64, ks), id1, kb > 0 || ks > 0);
          } else {
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
              umma_bf16(acc2, kmaj_desc(xb, 128, ks),
                        jb.y2_kmaj ? kmaj_desc(yb, 128, ks) : mnmaj_desc(yb, 64, ks), id2,
                        kb > 2 || ks > 0);
          }
          umma_commit(&empty[s]);
          last_bar = &empty[s];
          last_par = (it / kDualStages) & 1;
        }
        if (!ok) {
          *abort_flag = 1;
          break;
        }
        umma_commit(&acc_full[b]);
        last_bar = &acc_full[b];
        last_par = (tl >> 1) & 1;
      }
      if (last_bar) mbar_wait(last_bar, last_par);  // all issued MMAs are done
    }
  } else {
    // ------------------------------------------------ epilogue
    const int quad = warp & 3, half = warp >> 2;
    const int r = quad * 32 + lane;  // tile row = TMEM lane
    const uint32_t lane_tmem = tmem + ((quad * 32) << 16);
    const uint32_t scratch = smem_u32(smem) + kDualRing + warp * 2048;
    const size_t slot = size_t(p.BH) * p.TP;
    int tl = 0;
    for (int u = blockIdx.x; u < nunits; u += gridDim.x, ++tl) {
      const int tile = u / p.units, ui = u % p.units;
      const int nb = p.unit_nb[ui];
      const DualJob& jb = p.job[p.unit_job[ui]];
      const int bh = tile / p.NT, j = tile % p.NT, b = tl & 1;
      const int N = jb.N, c_beg = 128 * nb + 64 * half;  // this warp's 64 output columns
      const int t = j * 128 + r;
      const float* Gt = p.G + size_t(bh) * p.TP + j * 128;
      const float f = jb.fkind == 0 ? jb.scale * exp2f(Gt[r]) : exp2f(Gt[127] - Gt[r]);
      const size_t row = size_t(bh) * p.TP + t;
      const __nv_bfloat16* dsrc = jb.dot_src;
      // the row-dot partner, fetched coalesced before the MMAs are waited for
      uint4 dpre[2][4];
      if (dsrc) {
        const __nv_bfloat16* src = dsrc + (size_t(bh) * p.TP + j * 128 + quad * 32) * N + c_beg;
#pragma unroll
        for (int c = 0; c < 2; ++c) warp_fetch_block_bf16(src + 32 * c, N, dpre[c]);
      }
      const bool got =
          __all_sync(0xffffffffu, *abort_flag == 0 && mbar_wait(&acc_full[b], (tl >> 1) & 1));
      tc_fence_after();
      float dot = 0.f;
      if (got) {
        const uint32_t acc1 = lane_tmem + b * 256 + 64 * half, acc2 = acc1 + 128;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int col = c_beg + 32 * c;
          float a[32], bb[32];
          tmem_ld32x2(acc1 + 32 * c, a, acc2 + 32 * c, bb);
#pragma unroll
          for (int i = 0; i < 32; ++i) a[i] += f * bb[i];
          if (dsrc) {
            uint4 drow[4];
            warp_transpose_block_bf16(scratch, dpre[c], drow);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              float x[8];
              unpack_bf16x8(drow[q], x);
#pragma unroll
              for (int e = 0; e < 8; ++e) dot += x[e] * a[8 * q + e];
            }
          }
          if (jb.out_mode == 2) {
            const int b_ = bh / p.H, h = bh % p.H, t0 = j * 128 + quad * 32;
            const int nvalid = p.T - t0;
            const uint32_t valid =
                nvalid >= 32 ? 0xffffffffu : (nvalid <= 0 ? 0u : (1u << nvalid) - 1u);
            warp_store_block_bf16(scratch, a,
                                  static_cast<__nv_bfloat16*>(jb.out) +
                                      (size_t(b_) * p.T + t0) * jb.out_stride + size_t(h) * N + col,
                                  jb.out_stride, valid);
          } else if (jb.out_mode == 3) {
            warp_store_block_bf16(scratch, a,
                                  static_cast<__nv_bfloat16*>(jb.out) +
                                      (size_t(bh) * p.TP + j * 128 + quad * 32) * N + col,
                                  N, 0xffffffffu);
          } else {
            float4* dst = reinterpret_cast<float4*>(static_cast<float*>(jb.out) + row * N + col);
#pragma unroll
            for (int q = 0; q < 8; ++q)
              __stcs(dst + q, make_float4(a[4 * q], a[4 * q + 1], a[4 * q + 2], a[4 * q + 3]));
          }
        }
      }
      // hand the TMEM buffer back to the MMA issuer
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
      if (dsrc) dot_half[tl & 1][half][r] = dot;
      // join the two column halves of the row dot (and agree on stopping)
      if (named_bar_or(1, 256, !got)) {
        *abort_flag = 1;
        break;
      }
      if (dsrc && half == 0)
        jb.dG[nb * slot + row] = jb.dot_sign * (dot_half[tl & 1][0][r] + dot_half[tl & 1][1][r]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================ readout adjoint
struct ReadoutBwdParams {
  int BH, H, TP, NT, B;
  int per_head;                  // CTAs per head; gridDim.x = H * per_head
  const __nv_bfloat16* raw;      // [BH,TP,128]
  const __nv_bfloat16* dweights;  // [BH,TP,128]
  const float* lam;              // [BH,TP]
  __nv_bfloat16* draw;           // [BH,TP,128]
  float* dlam;                   // [BH,TP]
  float* dtab_part;              // [H * per_head, 128, 128]
};

// table | z | dc | p | dl (32 KiB each) | raw | dw staging (32 KiB each)
constexpr int kReadoutBwdSmem = 224 * 1024 + 1024;

// Persistent over the tiles of one head: CTA (h, split) handles tiles
// split, split + per_head, ... of head h and accumulates the table gradient in
// TMEM across them (one partial per CTA).  8 warps: warp w owns TMEM lane
// quadrant (w & 3) (token rows) and column half (w >> 2).  Per tile:
//   z = U(lam) raw, dc = U(lam) dw                  (registers -> bf16 smem)
//   logits = z Tab^T, dp = dc Tab^T                  (UMMA)
//   p = softmax(logits), dl = p o (dp - <p,dp>)     (registers; row halves joined in smem)
//   dz = dl Tab, coeff = p Tab, dTab += p^T dc + dl^T z   (UMMA)
//   draw = U(-lam) dz,  dlam = sum_p w_p [z x dz + dc x coeff]   (epilogue)
// The rotation terms use the on-chip z, dc and coeff, so no input is read twice.
// The raw and dweights tiles of the next tile are fetched by TMA into a staging
// area while the current tile computes.
__device__ __forceinline__ void readout_bwd_issue(uint8_t* smem, const CUtensorMap* mraw,
                                                  const CUtensorMap* mdw, const ReadoutBwdParams& p,
                                                  int h, int tile, uint64_t* bar) {
  const int b = tile / p.NT, j = tile % p.NT, bh = b * p.H + h;
  const int row0 = bh * p.TP + j * 128;
  mbar_expect_tx(bar, 65536);
  load_hist_tile(smem + 163840, mraw, row0, 0, 128, 128, bar);
  load_hist_tile(smem + 196608, mdw, row0, 0, 128, 128, bar);
}

__global__ void __launch_bounds__(256, 1)
    readout_bwd_kernel(const __grid_constant__ CUtensorMap map_tab,
                       const __grid_constant__ CUtensorMap map_raw,
                       const __grid_constant__ CUtensorMap map_dw, ReadoutBwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  __shared__ __align__(8) uint64_t bar_tab, bar_m1, bar_m2, bar_ld;
  __shared__ uint32_t tmem_base;
  __shared__ float xch[2][128];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, half = warp >> 2;
  const int r = quad * 32 + lane;
  const int h = blockIdx.x / p.per_head, split = blockIdx.x % p.per_head;
  const int ntiles = p.B * p.NT;
  if (tid == 0) {
    mbar_init(&bar_tab, 1);
    mbar_init(&bar_m1, 1);
    mbar_init(&bar_m2, 1);
    mbar_init(&bar_ld, 1);
    mbar_fence_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base, 512);
    tmem_relinquish();  // one allocation per CTA: let co-resident CTAs allocate
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();
  pdl_trigger();
  const uint32_t tmem = tmem_base;
  const uint32_t lane_tmem = tmem + ((quad * 32) << 16);
  const uint32_t sTab = smem_u32(smem), sZ = sTab + 32768, sDC = sTab + 65536,
                 sP = sTab + 98304, sDL = sTab + 131072;
  const uint32_t sRaw = sTab + 163840, sDw = sTab + 196608;
  bool ld_pending = false;  // elected thread: a staging load in flight
  if (tid == 0) {
    mbar_expect_tx(&bar_tab, 32768);
    load_hist_tile(smem, &map_tab, h * 128, 0, 128, 128, &bar_tab);
    if (split < ntiles) {
      readout_bwd_issue(smem, &map_raw, &map_dw, p, h, split, &bar_ld);
      ld_pending = true;
    }
  }
  bool ok = true;
  int it = 0;
  auto lam_of = [&](int tl) {
    const int bh_ = (tl / p.NT) * p.H + h;
    return p.lam[size_t(bh_) * p.TP + (tl % p.NT) * 128 + r];
  };
  float lam_next = split < ntiles ? lam_of(split) : 0.f;
  for (int tile = split; tile < ntiles; tile += p.per_head, ++it) {
    const int b = tile / p.NT, j = tile % p.NT, bh = b * p.H + h;
    const size_t row = size_t(bh) * p.TP + j * 128 + r;
    const float lam = lam_next;
    if (tile + p.per_head < ntiles) lam_next = lam_of(tile + p.per_head);
    if (!mbar_wait(&bar_ld, it & 1)) ok = false;
    if (tid == 0) ld_pending = false;
    // ---- z = U(lam) raw and dc = U(lam) dw for this thread's 64 columns
    {
      float z[64], dc[64];
#pragma unroll
      for (int q = 0; q < 8; ++q) unpack_bf16x8(ld_shared_v4(sRaw + half * 16384 + sw128(r, q)), z + 8 * q);
#pragma unroll
      for (int q = 0; q < 8; ++q) unpack_bf16x8(ld_shared_v4(sDw + half * 16384 + sw128(r, q)), dc + 8 * q);
#pragma unroll
      for (int i = 0; i < 64; i += 2) {
        float sn, cs;
        __sincosf(clock_phase(lam, 32 * half + i / 2), &sn, &cs);
        const float e = z[i], o = z[i + 1];
        z[i] = cs * e - sn * o;
        z[i + 1] = sn * e + cs * o;
        const float de = dc[i], dd = dc[i + 1];
        dc[i] = cs * de - sn * dd;
        dc[i + 1] = sn * de + cs * dd;
      }
      store_row64_bf16(sZ + half * 16384, r, z);
      store_row64_bf16(sDC + half * 16384, r, dc);
    }
    fence_async_smem();
    tc_fence_before();
    ok = __syncthreads_and(ok);
    tc_fence_after();
    if (!ok) break;
    // the staging area is free: fetch the next tile's inputs
    if (tid == 0 && tile + p.per_head < ntiles) {
      readout_bwd_issue(smem, &map_raw, &map_dw, p, h, tile + p.per_head, &bar_ld);
      ld_pending = true;
    }
    if (tid == 0) {
      if (it > 0 || mbar_wait(&bar_tab, 0)) {
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          umma_bf16(tmem, kmaj_desc(sZ, 128, ks), kmaj_desc(sTab, 128, ks),
                    make_idesc(128, 128, 0, 0), ks > 0);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          umma_bf16(tmem + 128, kmaj_desc(sDC, 128, ks), kmaj_desc(sTab, 128, ks),
                    make_idesc(128, 128, 0, 0), ks > 0);
        umma_commit(&bar_m1);
      } else {
        mbar_arrive(&bar_m1);
      }
    }
    __syncwarp();
    if (!mbar_wait(&bar_m1, it & 1)) ok = false;
    tc_fence_after();
    // ---- softmax over the 127 active slots, row split over two column halves
    float l[64], d[64];
    tmem_ld32(lane_tmem + half * 64, *reinterpret_cast<float(*)[32]>(l));
    tmem_ld32(lane_tmem + half * 64 + 32, *reinterpret_cast<float(*)[32]>(l + 32));
    tmem_ld32(lane_tmem + 128 + half * 64, *reinterpret_cast<float(*)[32]>(d));
    tmem_ld32(lane_tmem + 128 + half * 64 + 32, *reinterpret_cast<float(*)[32]>(d + 32));
    float mx = -1e30f;
#pragma unroll
    for (int i = 0; i < 64; ++i)
      if (half * 64 + i < 127) mx = fmaxf(mx, l[i]);
    xch[half][r] = mx;
    __syncthreads();
    mx = fmaxf(xch[0][r], xch[1][r]);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      l[i] = (half * 64 + i < 127) ? __expf(l[i] - mx) : 0.f;
      sum += l[i];
    }
    __syncthreads();
    xch[half][r] = sum;
    __syncthreads();
    const float inv = 1.f / (xch[0][r] + xch[1][r]);
    float pdp = 0.f;
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      l[i] *= inv;
      pdp += l[i] * d[i];
    }
    __syncthreads();
    xch[half][r] = pdp;
    __syncthreads();
    pdp = xch[0][r] + xch[1][r];
    store_row64_bf16(sP + half * 16384, r, l);
#pragma unroll
    for (int i = 0; i < 64; ++i) d[i] = l[i] * (d[i] - pdp);
    store_row64_bf16(sDL + half * 16384, r, d);
    fence_async_smem();
    tc_fence_before();
    ok = __syncthreads_and(ok);
    tc_fence_after();
    if (!ok) break;
    if (tid == 0) {
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)
        umma_bf16(tmem + 256, kmaj_desc(sDL, 128, ks), mnmaj_desc(sTab, 128, ks),
                  make_idesc(128, 128, 0, 1), ks > 0);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)
        umma_bf16(tmem, kmaj_desc(sP, 128, ks), mnmaj_desc(sTab, 128, ks),
                  make_idesc(128, 128, 0, 1), ks > 0);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)
        umma_bf16(tmem + 384, mnmaj_desc(sP, 128, ks), mnmaj_desc(sDC, 128, ks),
                  make_idesc(128, 128, 1, 1), (it > 0 || ks > 0) ? 1u : 0u);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)
        umma_bf16(tmem + 384, mnmaj_desc(sDL, 128, ks), mnmaj_desc(sZ, 128, ks),
                  make_idesc(128, 128, 1, 1), 1);
      umma_commit(&bar_m2);
    }
    __syncwarp();
    if (!mbar_wait(&bar_m2, it & 1)) ok = false;
    tc_fence_after();
    // ---- draw = U(-lam) dz, dlam from the rotations (z, dc from smem, coeff from TMEM)
    {
      float dz[64], cf[64];
      tmem_ld32(lane_tmem + 256 + half * 64, *reinterpret_cast<float(*)[32]>(dz));
      tmem_ld32(lane_tmem + 256 + half * 64 + 32, *reinterpret_cast<float(*)[32]>(dz + 32));
      tmem_ld32(lane_tmem + half * 64, *reinterpret_cast<float(*)[32]>(cf));
      tmem_ld32(lane_tmem + half * 64 + 32, *reinterpret_cast<float(*)[32]>(cf + 32));
      float dl = 0.f;
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8) {
        float z[8], dc[8];
        unpack_bf16x8(ld_shared_v4(sZ + half * 16384 + sw128(r, c8)), z);
        unpack_bf16x8(ld_shared_v4(sDC + half * 16384 + sw128(r, c8)), dc);
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          const int i = 8 * c8 + e;
          const int pair = 32 * half + i / 2;
          float sn, cs;
          __sincosf(clock_phase(lam, pair), &sn, &cs);
          const float de = dz[i], dd = dz[i + 1];
          dl += (pair * kTwoPiOver127) *
                (-de * z[e + 1] + dd * z[e] + dc[e] * cf[i + 1] - dc[e + 1] * cf[i]);
          dz[i] = cs * de + sn * dd;
          dz[i + 1] = -sn * de + cs * dd;
        }
      }
      __nv_bfloat16* dst = p.draw + row * 128 + half * 64;
      store_bf16x32_global(dst, dz);
      store_bf16x32_global(dst + 32, dz + 32);
      __syncthreads();
      xch[half][r] = dl;
      __syncthreads();
      if (half == 0) p.dlam[row] = xch[0][r] + xch[1][r];
    }
    tc_fence_before();
    ok = __syncthreads_and(ok);  // smem tiles and TMEM are reused by the next tile
    tc_fence_after();
    if (!ok) break;
  }
  if (tid == 0 && ld_pending) mbar_wait(&bar_ld, it & 1);  // error path: let it land
  // this CTA's partial table gradient: thread (quad, half) owns slot row r, 64 columns
  if (ok && it > 0) {
    float* dst = p.dtab_part + size_t(blockIdx.x) * 16384 + r * 128 + half * 64;
#pragma unroll 1
    for (int c = 0; c < 2; ++c) {
      float v[32];
      tmem_ld32(lane_tmem + 384 + half * 64 + 32 * c, v);
      float4* d4 = reinterpret_cast<float4*>(dst + 32 * c);
#pragma unroll
      for (int q = 0; q < 8; ++q)
        d4[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Readout table of the chunked op in the kernels' bf16 layout, last row zero:
//   tab[h][r][m] = sum_{k < 127} R[h][r][k] Phi[k][m]  (r < 127),  tab[h][127][:] = 0,
// the product Table_h = R_h Phi of the reference (ops/chunk.py:281) rounded once
// to bf16.  One CTA per (h, r), thread m; fixed-order fp32 sums.
__global__ void __launch_bounds__(128) readout_table_kernel(const float* R, const float* phi,
                                                            __nv_bfloat16* tab) {
  pdl_wait();
  pdl_trigger();
  const int h = blockIdx.x, r = blockIdx.y, m = threadIdx.x;
  __shared__ float row[128];
  if (r < 127 && m < 127) row[m] = R[(size_t(h) * 127 + r) * 127 + m];
  __syncthreads();
  float acc = 0.f;
  if (r < 127) {
    // loads issued 16 at a time (the basis comes from L2), then a fixed-order sum
#pragma unroll 16
    for (int k = 0; k < 127; ++k) acc = fmaf(row[k], __ldg(phi + k * 128 + m), acc);
  }
  tab[(size_t(h) * 128 + r) * 128 + m] = __float2bfloat16_rn(acc);
}

// Readout gradient from the table gradient (the adjoint of the product above):
//   dR[h][r][k] = sum_{m < 128} dtab[h][r][m] Phi[k][m],  r, k < 127,
// with phiT = Phi^T [128][127].  One CTA per (h, r), thread k; fixed-order sums.
__global__ void __launch_bounds__(128) readout_grad_kernel(const float* dtab, const float* phiT,
                                                           float* dR) {
  pdl_wait();
  pdl_trigger();
  const int h = blockIdx.x, r = blockIdx.y, k = threadIdx.x;
  __shared__ float row[128];
  row[k] = dtab[(size_t(h) * 128 + r) * 128 + k];
  __syncthreads();
  if (k < 127) {
    float acc = 0.f;
#pragma unroll 16
    for (int m = 0; m < 128; ++m) acc = fmaf(row[m], __ldg(phiT + m * 127 + k), acc);
    dR[(size_t(h) * 127 + r) * 127 + k] = acc;
  }
}

// Fixed-order reduction of the per-CTA table gradients:
// dtab[h][r][m] = sum_{s < per_head} part[h * per_head + s][r][m],
// and, with dR given, the readout gradient row r < 127 from the reduced row
// (the sums of readout_grad_kernel).
__global__ void __launch_bounds__(128) dtable_reduce_kernel(const float* part, float* dtab,
                                                            int per_head, const float* phiT,
                                                            float* dR) {
  pdl_wait();
  pdl_trigger();
  const int h = blockIdx.x, r = blockIdx.y, m = threadIdx.x;
  __shared__ float row[128];
  float s0 = 0.f, s1 = 0.f;
  int k = 0;
  for (; k + 1 < per_head; k += 2) {
    s0 += part[(size_t(h) * per_head + k) * 16384 + r * 128 + m];
    s1 += part[(size_t(h) * per_head + k + 1) * 16384 + r * 128 + m];
  }
  if (k < per_head) s0 += part[(size_t(h) * per_head + k) * 16384 + r * 128 + m];
  const float s = s0 + s1;
  dtab[(size_t(h) * 128 + r) * 128 + m] = s;
  if (dR == nullptr || r >= 127) return;
  row[m] = s;
  __syncthreads();
  if (m < 127) {
    float acc = 0.f;
#pragma unroll 16
    for (int c = 0; c < 128; ++c) acc = fmaf(row[c], __ldg(phiT + c * 127 + m), acc);
    dR[(size_t(h) * 127 + r) * 127 + m] = acc;
  }
}

// Fixed-order column sums of a [rows, cols] partial matrix: out[c] = sum_r part[r][c].
// 1024 threads: 32 columns x 32 row lanes, each lane with 4 independent accumulators.
// Columns c >= split go to out_hi[c - split] instead of out[c].
__global__ void __launch_bounds__(1024) column_sum_kernel(const float* part, float* out, int rows,
                                                          int cols, const float* part2 = nullptr,
                                                          float* out2 = nullptr,
                                                          int split = 0x7fffffff,
                                                          float* out_hi = nullptr) {
  __shared__ float acc[32][33];
  pdl_wait();
  pdl_trigger();
  if (blockIdx.y == 1) {  // second (part, out) pair
    part = part2;
    out = out2;
  }
  const int c = blockIdx.x * 32 + (threadIdx.x & 31), lane_r = threadIdx.x >> 5;
  float s = 0.f;
  if (c < cols) {
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
    int r = lane_r;
    for (; r + 96 < rows; r += 128) {
      s0 += part[size_t(r) * cols + c];
      s1 += part[size_t(r + 32) * cols + c];
      s2 += part[size_t(r + 64) * cols + c];
      s3 += part[size_t(r + 96) * cols + c];
    }
    for (; r < rows; r += 32) s0 += part[size_t(r) * cols + c];
    s = (s0 + s1) + (s2 + s3);
  }
  acc[lane_r][threadIdx.x & 31] = s;
  __syncthreads();
  if (threadIdx.x < 32 && c < cols) {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) t += acc[i][threadIdx.x];
    if (c < split) out[c] = t;
    else out_hi[c - split] = t;
  }
}

}  // namespace cyfa
