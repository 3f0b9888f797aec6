// Chunked scalar-gated linear attention (ScalarGatedLA) forward on tcgen05.
//
// One pass computes, per (batch, head) and 128-token tile j (two of the
// reference's 64-token chunks; the result does not depend on the tile size),
//   S_{j+1} = 2^{G_L} S_j + K_j^T (V_j o 2^{G_L - G_t})                  (state scan)
//   o_t     = scale [2^{G_t} q_t S_j + sum_{s<=t} 2^{G_t - G_s} (q_t.k_s) v_s]  (tile output)
// with G the log2 in-tile cumsum of the gate.  This replaces the reference's
// state_forward (cyclic_flow_attention/ops/chunk_h.py:10-343) and output_forward /
// first_readout (ops/chunk_o.py:10-613, ops/chunk_readout.py:792-991).
//
// state_scan_kernel: one CTA per (bh, 128-row K slice, 64-column V slice).
//   Tiles stream through a 3-stage TMA ring; the V tile is rescaled in place by
//   the 128 threads (one token row each); one thread issues the 128x64x128 UMMA
//   into a double-buffered TMEM accumulator; each thread keeps its state row
//   (64 fp32) in registers, stores it as bf16 history S_j and adds the update.
//   REVERSE runs the same recurrence backwards for the state adjoint
//   H_j = 2^{G_L} H_{j+1} + Q_j^T (dO_j o scale 2^{G_t}) and also emits the
//   per-tile gate boundary term <S_{j+1}, H_{j+1}>.
// tile_fwd_kernel (pass 2) / tile_fwd_ro_kernel (pass 1): one CTA per (bh, tile,
//   128-column V slice); all GEMMs of the tile on tcgen05 (Q K^T, Q S_j, P V),
//   accumulators in TMEM, operands staged by TMA.  Pass 1's epilogue applies the
//   softmax slot readout (ops/chunk.py:320-331): z = U(lam) raw, logits =
//   z Table^T, p = softmax over the 127 active slots, coeff = p Table, weights =
//   U(-lam) coeff, with both table products on tcgen05 and the rotations in
//   registers.
#include "cyfa_common.cuh"
#include "phase.cuh"

namespace cyfa {

enum RowMode : int { kRows2D = 0, kPublic4D = 1 };

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// Loads `cols` columns (from c0) of the 128-token tile j of head-row bh as
// cols/64 swizzled blocks of [128 x 64] (16 KiB apart).  2-D maps index rows
// bh*TP + t; public 4-D maps are {D, H, T, B} (rows past T read as zeros).
__device__ __forceinline__ void load_token_tile(uint8_t* dst, const CUtensorMap* map, int mode,
                                                int bh, int H, int TP, int j, int c0, int cols,
                                                uint64_t* bar) {
  for (int cb = 0; cb < cols / 64; ++cb) {
    if (mode == kRows2D)
      tma_load_2d(dst + cb * 16384, map, bar, c0 + 64 * cb, bh * TP + j * 128);
    else
      tma_load_4d(dst + cb * 16384, map, bar, c0 + 64 * cb, bh % H, j * 128, bh / H);
  }
}

// Loads `cols` columns (from c0) of R history rows starting at row0 as cols/64
// blocks of [R x 64] (R*128 bytes apart).
__device__ __forceinline__ void load_hist_tile(uint8_t* dst, const CUtensorMap* map, int row0,
                                               int c0, int cols, int R, uint64_t* bar) {
  for (int cb = 0; cb < cols / 64; ++cb)
    tma_load_2d(dst + cb * R * 128, map, bar, c0 + 64 * cb, row0);
}

__device__ __forceinline__ void store_bf16x32_global(__nv_bfloat16* dst, const float* v) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int c = 0; c < 4; ++c)
    d[c] = make_uint4(pack_bf16(v[8 * c], v[8 * c + 1]), pack_bf16(v[8 * c + 2], v[8 * c + 3]),
                      pack_bf16(v[8 * c + 4], v[8 * c + 5]), pack_bf16(v[8 * c + 6], v[8 * c + 7]));
}

// ============================================================ state scan
struct ScanParams {
  int BH, H, TP, NT;
  int DK, DV;
  int k_mode, v_mode;
  const float* G;           // [BH, TP] log2 in-tile gate cumsum
  const float* init;        // [BH, DK, DV] fp32 or null
  __nv_bfloat16* hist;      // [BH, NT, DK, DV]: state entering each tile
  float* last;              // [BH, DK, DV]: final state (forward) / initial-state adjoint
  float scale;              // reverse: scale of dO
  __nv_bfloat16* last_bf;   // forward: bf16 copy of the final state [BH, DK, DV], or null
  float* bpart;             // reverse: [BH, NT, nsub, 4] partial boundary terms
  const float* final_f32;   // reverse: the forward final state [BH, DK, DV] fp32, or null
  // Segmented scan (tiles split into nseg segments of seg_tiles, grid z = V slices
  // x segments).  summary != 0: each segment runs from zero (the segment holding
  // the sequence's first tile in scan order from `init`), writes only its end
  // state to seg_out [nseg, BH, DK, DV], no history, no boundary terms.
  // summary == 0 with nseg > 1: segment s starts from seg_init[s] (the carry
  // formed by scan_carry_kernel) unless it holds the first tile.
  int nseg, seg_tiles, summary;
  const float* seg_init;
  float* seg_out;
};

// Ring of the scan: forward stages hold the K tile (32 KiB) and the V tile
// (16 KiB); reverse stages also hold the forward state S_{j+1} slice (16 KiB)
// that the boundary term of tile j pairs with.
template <bool REVERSE>
struct ScanRing {
  static constexpr int stages = REVERSE ? 3 : 4;
  static constexpr int stage_bytes = (REVERSE ? 64 : 48) * 1024;
};
constexpr int kScanRingBytes = 192 * 1024;
static_assert(ScanRing<false>::stages * ScanRing<false>::stage_bytes <= kScanRingBytes &&
                  ScanRing<true>::stages * ScanRing<true>::stage_bytes <= kScanRingBytes,
              "scan ring");
// ring + 4 KiB staging per consumer warp (coalesced history traffic) + alignment
constexpr int kScanSmem = kScanRingBytes + 4 * 4096 + 1024;
constexpr int kScanBufs = 4;                // TMEM update buffers of 64 columns

// OR of v over the `n` threads of named barrier `id` (every one of them gets it).
__device__ __forceinline__ bool named_bar_or(int id, int n, bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, %2, %3, p;\n"
      " selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"(v ? 1u : 0u), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}

// Chunk-state scan, warp-specialised.  One CTA owns rows dk0..dk0+127 and
// columns dv0..dv0+63 of the state of one (b, h); 320 threads in five roles that
// hand tiles to each other through mbarriers only:
//   warp 8, lane 0 (producer): TMA loads of each tile's K/V operands (and, in
//     REVERSE, the forward state slice S_{j+1}) into a ring of stages; a stage is
//     refilled once the UMMA (and, in REVERSE, the consumers) of its previous
//     tile are done with it;
//   warps 4-7 (scalers): scale the tile's V rows by its gate factor in shared
//     memory, then signal `scaled`;
//   warp 9, lane 0 (MMA issuer): U = K^T (V o f) into one of kScanBufs TMEM
//     buffers once the consumers have released it;
//   warps 0-3 (consumers): thread r keeps state row r in registers, stores the
//     state entering each tile (bf16 history) and applies S = 2^{G_last} S + U.
// The updates U do not depend on the state, so producer, scalers and issuer run
// up to kScanBufs tiles ahead of the serial recurrence.
// REVERSE walks the tiles backwards with f = scale 2^{G_t} (adjoint scan) and
// also forms the boundary partials <S_{j+1}, H_{j+1}> from the forward history
// (map_f, rows of S_{j+1} for j + 1 < NT) or the forward final state (map_ff),
// both bf16 and brought in by the producer with the tile's operands.
constexpr int kScanThreads = 320;

template <bool REVERSE>
__global__ void __launch_bounds__(kScanThreads, 1)
    state_scan_kernel(const __grid_constant__ CUtensorMap map_k,
                      const __grid_constant__ CUtensorMap map_v,
                      const __grid_constant__ CUtensorMap map_f,
                      const __grid_constant__ CUtensorMap map_ff, ScanParams p) {
  constexpr int kScanStages = ScanRing<REVERSE>::stages;
  constexpr int kScanStageBytes = ScanRing<REVERSE>::stage_bytes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  __shared__ __align__(8) uint64_t full[kScanStages];
  __shared__ __align__(8) uint64_t scaled[kScanStages];
  __shared__ __align__(8) uint64_t f_free[kScanStages];
  __shared__ __align__(8) uint64_t mma_done[kScanBufs];
  __shared__ __align__(8) uint64_t tmem_free[kScanBufs];
  __shared__ uint32_t tmem_base;
  __shared__ int s_abort;
  volatile int* abort_flag = &s_abort;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nvs = p.DV / 64;
  const int bh = blockIdx.x, dk0 = blockIdx.y * 128, vs = blockIdx.z % nvs, seg = blockIdx.z / nvs;
  const int dv0 = vs * 64;
  const int NT = p.NT;
  // this CTA's tiles [t0, t1), walked backwards in REVERSE
  const int t0 = seg * p.seg_tiles, t1 = min(t0 + p.seg_tiles, NT);
  const int nloc = t1 > t0 ? t1 - t0 : 0;
  // the segment holding the first tile in scan order starts from `init`
  const bool first_seg = REVERSE ? (t1 == NT) : (t0 == 0);
  // the segment holding the last tile in scan order writes the final outputs
  const bool last_seg = REVERSE ? (t0 == 0) : (t1 == NT);
  const bool with_f = REVERSE && !p.summary;  // boundary terms need S_{j+1}
  static_assert(kScanStages <= kScanBufs, "stage reuse relies on mma_done parity");

  if (tid == 0) {
    for (int s = 0; s < kScanStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&scaled[s], 4);
      mbar_init(&f_free[s], 4);
    }
    for (int b = 0; b < kScanBufs; ++b) {
      mbar_init(&mma_done[b], 1);
      mbar_init(&tmem_free[b], 4);
    }
    s_abort = 0;
    mbar_fence_init();
    prefetch_tmap(&map_k);
    prefetch_tmap(&map_v);
    if (REVERSE) {
      prefetch_tmap(&map_f);
      prefetch_tmap(&map_ff);
    }
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base, 64 * kScanBufs);
    tmem_relinquish();  // one allocation per CTA: let co-resident CTAs allocate
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();
  pdl_trigger();
  const uint32_t tmem = tmem_base;
  auto tile_of = [&](int idx) { return REVERSE ? t1 - 1 - idx : t0 + idx; };
  const float* Gbh = p.G + size_t(bh) * p.TP;

  if (warp == 8) {
    // ------------------------------------------------ producer
    if (lane == 0) {
      int issued = 0;
      for (int idx = 0; idx < nloc; ++idx) {
        if (*abort_flag) break;
        const int s = idx % kScanStages, j = tile_of(idx);
        if (idx >= kScanStages) {
          const int prev = idx - kScanStages;  // previous tile of this stage
          bool ok = mbar_wait(&mma_done[prev % kScanBufs], (prev / kScanBufs) & 1);
          if (with_f && ok) ok = mbar_wait(&f_free[s], (prev / kScanStages) & 1);
          if (!ok) {
            *abort_flag = 1;
            break;
          }
        }
        uint8_t* st = smem + s * kScanStageBytes;
        mbar_expect_tx(&full[s], with_f ? 65536 : 49152);
        load_token_tile(st, &map_k, p.k_mode, bh, p.H, p.TP, j, dk0, 128, &full[s]);
        load_token_tile(st + 32768, &map_v, p.v_mode, bh, p.H, p.TP, j, dv0, 64, &full[s]);
        if (with_f) {
          if (j + 1 < NT)
            tma_load_2d(st + 49152, &map_f, &full[s], dv0, (bh * NT + j + 1) * p.DK + dk0);
          else
            tma_load_2d(st + 49152, &map_ff, &full[s], dv0, bh * p.DK + dk0);
        }
        issued = idx + 1;
      }
      // every issued copy lands before shared memory goes away
      for (int idx = issued > kScanStages ? issued - kScanStages : 0; idx < issued; ++idx)
        mbar_wait(&full[idx % kScanStages], (idx / kScanStages) & 1);
    }
  } else if (warp == 9) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = make_idesc(128, 64, 1, 1);
      int last_commit = -1;
      for (int idx = 0; idx < nloc; ++idx) {
        if (*abort_flag) break;
        const int s = idx % kScanStages, b = idx % kScanBufs;
        bool ok = mbar_wait(&scaled[s], (idx / kScanStages) & 1);
        if (ok && idx >= kScanBufs) ok = mbar_wait(&tmem_free[b], ((idx / kScanBufs) - 1) & 1);
        if (!ok) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t kb = smem_u32(smem + s * kScanStageBytes), vb = kb + 32768;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          umma_bf16(tmem + b * 64, mnmaj_desc(kb, 128, ks), mnmaj_desc(vb, 128, ks), idesc,
                    ks > 0);
        umma_commit(&mma_done[b]);
        last_commit = idx;
      }
      if (last_commit >= 0)
        mbar_wait(&mma_done[last_commit % kScanBufs], (last_commit / kScanBufs) & 1);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------ scalers
    const int srow = tid - 128;
    float gt_n = 0.f, gl_n = 0.f;
    if (nloc > 0) {
      gt_n = Gbh[size_t(tile_of(0)) * 128 + srow];
      gl_n = Gbh[size_t(tile_of(0)) * 128 + 127];
    }
    for (int idx = 0; idx < nloc; ++idx) {
      const int s = idx % kScanStages;
      const float gt = gt_n, gl = gl_n;
      if (idx + 1 < nloc) {
        gt_n = Gbh[size_t(tile_of(idx + 1)) * 128 + srow];
        gl_n = Gbh[size_t(tile_of(idx + 1)) * 128 + 127];
      }
      const float f = REVERSE ? p.scale * exp2f(gt) : exp2f(gl - gt);
      const bool got =
          __all_sync(0xffffffffu, *abort_flag == 0 && mbar_wait(&full[s], (idx / kScanStages) & 1));
      if (!got) {
        *abort_flag = 1;
        break;
      }
      const uint32_t vb = smem_u32(smem + s * kScanStageBytes + 32768);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint32_t a = vb + sw128(srow, c);
        float x[8];
        unpack_bf16x8(ld_shared_v4(a), x);
        st_shared_v4(a, pack_bf16(x[0] * f, x[1] * f), pack_bf16(x[2] * f, x[3] * f),
                     pack_bf16(x[4] * f, x[5] * f), pack_bf16(x[6] * f, x[7] * f));
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&scaled[s]);
    }
  } else {
    // ------------------------------------------------ consumers: the recurrence
    float S[64];
    const size_t row_off = (size_t(bh) * p.DK + dk0 + tid) * p.DV + dv0;
    const float* init = first_seg ? p.init
                        : (p.summary ? nullptr
                                     : p.seg_init + size_t(seg) * p.BH * p.DK * p.DV);
    if (init) {
      const float4* src = reinterpret_cast<const float4*>(init + row_off);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float4 x = src[i];
        S[4 * i] = x.x;
        S[4 * i + 1] = x.y;
        S[4 * i + 2] = x.z;
        S[4 * i + 3] = x.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 64; ++i) S[i] = 0.f;
    }
    const uint32_t lane_tmem = tmem + ((warp * 32) << 16);
    const uint32_t scratch = smem_u32(smem) + kScanStages * kScanStageBytes + warp * 4096;
    const int nsub = gridDim.y * nvs, sub = blockIdx.y * nvs + vs;
    bool ok = true;
    // the gate total of the next tile is loaded one iteration ahead
    float gl_next = nloc > 0 ? Gbh[size_t(tile_of(0)) * 128 + 127] : 0.f;
    for (int idx = 0; idx < nloc; ++idx) {
      const int j = tile_of(idx), b = idx % kScanBufs;
      const float gl = gl_next;
      if (idx + 1 < nloc) gl_next = Gbh[size_t(tile_of(idx + 1)) * 128 + 127];
      // state entering tile j (forward) / adjoint leaving tile j (reverse)
      if (!p.summary) {
        uint4 packed[8];
#pragma unroll
        for (int c = 0; c < 8; ++c)
          packed[c] = make_uint4(pack_bf16(S[8 * c], S[8 * c + 1]), pack_bf16(S[8 * c + 2], S[8 * c + 3]),
                                 pack_bf16(S[8 * c + 4], S[8 * c + 5]),
                                 pack_bf16(S[8 * c + 6], S[8 * c + 7]));
        warp_store_rows128(scratch, packed,
                           p.hist + ((size_t(bh) * NT + j) * p.DK + dk0 + warp * 32) * p.DV + dv0,
                           p.DV);
      }
      bool got = __all_sync(0xffffffffu, mbar_wait(&mma_done[b], (idx / kScanBufs) & 1));
      if (with_f) {
        // <S_{j+1}, H_{j+1}> over this CTA's slice; S holds H_{j+1} until the update
        const int s = idx % kScanStages;
        got = got && __all_sync(0xffffffffu, mbar_wait(&full[s], (idx / kScanStages) & 1));
        float dot = 0.f;
        if (got && j + 1 == NT && p.final_f32) {
          // the last tile pairs with the final state, which exists in fp32: its
          // boundary term cancels against the key rows' dots of the whole tile, so
          // the bf16 copy's rounding would dominate it when the final state's
          // adjoint is large
          const float4* fs = reinterpret_cast<const float4*>(p.final_f32 + row_off);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float4 x = fs[i];
            dot += x.x * S[4 * i] + x.y * S[4 * i + 1] + x.z * S[4 * i + 2] + x.w * S[4 * i + 3];
          }
        } else if (got) {
          const uint32_t fb = smem_u32(smem + s * kScanStageBytes + 49152);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            float x[8];
            unpack_bf16x8(ld_shared_v4(fb + sw128(tid, c)), x);
#pragma unroll
            for (int e = 0; e < 8; ++e) dot += x[e] * S[8 * c + e];
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        // one partial per warp: bpart[bh][j][sub][warp]
        if (lane == 0 && got) p.bpart[((size_t(bh) * NT + j) * nsub + sub) * 4 + warp] = dot;
        __syncwarp();
        if (lane == 0) mbar_arrive(&f_free[s]);
      }
      tc_fence_after();
      if (got) {
        const float gamma = exp2f(gl);
        float U[32];
        tmem_ld32(lane_tmem + b * 64, U);
#pragma unroll
        for (int i = 0; i < 32; ++i) S[i] = S[i] * gamma + U[i];
        tmem_ld32(lane_tmem + b * 64 + 32, U);
#pragma unroll
        for (int i = 0; i < 32; ++i) S[32 + i] = S[32 + i] * gamma + U[i];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tmem_free[b]);
      if (!got || __any_sync(0xffffffffu, *abort_flag != 0)) {
        ok = false;
        *abort_flag = 1;
        break;
      }
    }
    // a summary pass: the segment's end state, for scan_carry_kernel
    if (ok && p.summary) {
      float4* dst = reinterpret_cast<float4*>(p.seg_out + size_t(seg) * p.BH * p.DK * p.DV + row_off);
#pragma unroll
      for (int i = 0; i < 16; ++i)
        dst[i] = make_float4(S[4 * i], S[4 * i + 1], S[4 * i + 2], S[4 * i + 3]);
    }
    // the final state (forward) / initial-state adjoint (reverse)
    if (ok && !p.summary && last_seg && p.last) {
      float4* dst = reinterpret_cast<float4*>(p.last + row_off);
#pragma unroll
      for (int i = 0; i < 16; ++i)
        dst[i] = make_float4(S[4 * i], S[4 * i + 1], S[4 * i + 2], S[4 * i + 3]);
    }
    if (!REVERSE && ok && !p.summary && last_seg && p.last_bf) {
      uint4 packed[8];
#pragma unroll
      for (int c = 0; c < 8; ++c)
        packed[c] = make_uint4(pack_bf16(S[8 * c], S[8 * c + 1]), pack_bf16(S[8 * c + 2], S[8 * c + 3]),
                               pack_bf16(S[8 * c + 4], S[8 * c + 5]),
                               pack_bf16(S[8 * c + 6], S[8 * c + 7]));
      warp_store_rows128(scratch, packed,
                         p.last_bf + (size_t(bh) * p.DK + dk0 + warp * 32) * p.DV + dv0, p.DV);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 64 * kScanBufs);
  }
}

// Carries of the segmented scan (one thread per 4 state elements of one (b, h)):
// the state entering each segment from the summaries E_s of the segments before
// it (forward) or after it (reverse):
//   forward  C_1 = E_0,      C_{s+1} = Gamma_s C_s + E_s
//   reverse  D_{n-2} = E_{n-1}, D_{s-1} = Gamma_s D_s + E_s
// Gamma_s = the product over the segment's tiles of their decay 2^{G_last},
// formed in the scan's own order.  Writes seg_init[s] for every segment but the
// one holding the first tile.
constexpr int kScanCarryMaxSegs = 160;

template <bool REVERSE>
__global__ void __launch_bounds__(256) scan_carry_kernel(const float* G, int TP, int NT, int BH,
                                                         int elems, int nseg, int seg_tiles,
                                                         const float* seg_out, float* seg_init) {
  __shared__ float s_gamma[kScanCarryMaxSegs];
  pdl_wait();
  pdl_trigger();
  const int bh = blockIdx.y;
  const float* Gbh = G + size_t(bh) * TP;
  // Gamma_s of every segment, one thread each (the tile decays read in parallel)
  for (int s = threadIdx.x; s < nseg; s += blockDim.x) {
    float gm = 1.f;
    const int a = s * seg_tiles, b = min(a + seg_tiles, NT);
    if (REVERSE)
      for (int j = b - 1; j >= a; --j) gm *= exp2f(__ldg(Gbh + size_t(j) * 128 + 127));
    else
      for (int j = a; j < b; ++j) gm *= exp2f(__ldg(Gbh + size_t(j) * 128 + 127));
    s_gamma[s] = gm;
  }
  __syncthreads();
  const int e = (blockIdx.x * 256 + threadIdx.x) * 4;
  if (e >= elems) return;
  const size_t stride = size_t(BH) * elems, base = size_t(bh) * elems + e;
  auto gamma = [&](int s) { return s_gamma[s]; };
  const int first = REVERSE ? nseg - 1 : 0;
  float4 c = *reinterpret_cast<const float4*>(seg_out + first * stride + base);
  for (int k = 1; k < nseg; ++k) {
    const int s = REVERSE ? nseg - 1 - k : k;
    *reinterpret_cast<float4*>(seg_init + s * stride + base) = c;
    if (k + 1 < nseg) {
      const float gm = gamma(s);
      const float4 x = *reinterpret_cast<const float4*>(seg_out + s * stride + base);
      c = make_float4(c.x * gm + x.x, c.y * gm + x.y, c.z * gm + x.z, c.w * gm + x.w);
    }
  }
}

// ============================================================ tile output
struct TileFwdParams {
  int BH, H, TP, NT, T;
  int DV;          // full value width (public output stride)
  int v_mode;      // token-row mode of V
  int o_mode;      // 0: raw [BH, TP, 128] bf16 (pass 1); 1: public o [B, T, H, DV] bf16
  const float* G;  // [BH, TP]
  const float* lam;  // [BH, TP] clock (READOUT)
  float scale;
  __nv_bfloat16* out;
  __nv_bfloat16* weights;  // READOUT: [BH, TP, 128]
};

// Pass 2's output tile (queries = the readout weights, DK = 128), two CTAs per
// SM: V is loaded into the S region once Q S_j is done, the output staging uses
// the Q region, and P V accumulates into the Q K^T columns of TMEM (256 columns).
constexpr int kTileFwdSmem = 3 * 128 * 256 + 1024;

// 8 warps: warp w owns TMEM lane quadrant (w & 3) (token rows 32(w&3)..+31) and
// column half (w >> 2) of every 128-column accumulator.
__global__ void __launch_bounds__(256, 1)
    tile_fwd_kernel(const __grid_constant__ CUtensorMap map_q,
                    const __grid_constant__ CUtensorMap map_k,
                    const __grid_constant__ CUtensorMap map_v,
                    const __grid_constant__ CUtensorMap map_s, TileFwdParams p) {
  constexpr int DK = 128;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  constexpr int kQ = 0, kK = DK * 256, kS = 2 * DK * 256;
  __shared__ __align__(8) uint64_t bar_in, bar_v, bar_m[3];
  __shared__ uint32_t tmem_base;
  __shared__ float Gs[128];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, half = warp >> 2;
  const int r = quad * 32 + lane;
  const int bh = blockIdx.x / p.NT, j = blockIdx.x % p.NT, dv0 = blockIdx.y * 128;

  if (tid == 0) {
    mbar_init(&bar_in, 1);
    mbar_init(&bar_v, 1);
    for (int i = 0; i < 3; ++i) mbar_init(&bar_m[i], 1);
    mbar_fence_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base, 256);
    tmem_relinquish();  // one allocation per CTA: let co-resident CTAs allocate
  }
  pdl_wait();
  if (tid < 128) Gs[tid] = p.G[size_t(bh) * p.TP + j * 128 + tid];
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_trigger();
  const uint32_t tmem = tmem_base;
  const uint32_t lane_tmem = tmem + ((quad * 32) << 16);
  const uint32_t sQ = smem_u32(smem + kQ), sK = smem_u32(smem + kK), sS = smem_u32(smem + kS);
  bool ok = true;

  if (tid == 0) {
    mbar_expect_tx(&bar_in, 3 * DK * 256);
    load_token_tile(smem + kQ, &map_q, kRows2D, bh, p.H, p.TP, j, 0, DK, &bar_in);
    load_token_tile(smem + kK, &map_k, kRows2D, bh, p.H, p.TP, j, 0, DK, &bar_in);
    load_hist_tile(smem + kS, &map_s, (bh * p.NT + j) * DK, dv0, 128, DK, &bar_in);
    if (mbar_wait(&bar_in, 0)) {
      tc_fence_after();
      // S_qk = Q K^T -> TMEM[0,128); O_inter = Q S_j -> TMEM[128,256)
#pragma unroll 4
      for (int ks = 0; ks < DK / 16; ++ks)
        umma_bf16(tmem, kmaj_desc(sQ, 128, ks), kmaj_desc(sK, 128, ks), make_idesc(128, 128, 0, 0),
                  ks > 0);
      umma_commit(&bar_m[0]);
#pragma unroll 4
      for (int ks = 0; ks < DK / 16; ++ks)
        umma_bf16(tmem + 128, kmaj_desc(sQ, 128, ks), mnmaj_desc(sS, DK, ks),
                  make_idesc(128, 128, 0, 1), ks > 0);
      umma_commit(&bar_m[1]);
      // V into the S region once Q S_j has read it
      if (mbar_wait(&bar_m[1], 0)) {
        mbar_expect_tx(&bar_v, 32768);
        load_token_tile(smem + kS, &map_v, p.v_mode, bh, p.H, p.TP, j, dv0, 128, &bar_v);
      } else {
        mbar_arrive(&bar_v);
      }
    } else {
      mbar_arrive(&bar_m[0]);
      mbar_arrive(&bar_m[1]);
      mbar_arrive(&bar_v);
    }
  }
  const float gt = Gs[r];
  __syncwarp();
  // ---- P = mask(S_qk o 2^{G_t - G_s}) -> bf16, K-major A operand in the K region
  if (!mbar_wait(&bar_m[0], 0)) ok = false;
  tc_fence_after();
  if (ok) {
#pragma unroll 1
    for (int c = 0; c < 2; ++c) {
      const int col0 = half * 64 + 32 * c;
      float v[32];
      tmem_ld32(lane_tmem + col0, v);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int s_ = col0 + i;
        v[i] = s_ <= r ? v[i] * exp2f(gt - Gs[s_]) : 0.f;
      }
      store_row32_bf16(sK + half * 16384, r, c * 4, v);
    }
  }
  fence_async_smem();
  tc_fence_before();
  ok = __syncthreads_and(ok);
  tc_fence_after();
  if (tid == 0) {
    const bool vok = ok && mbar_wait(&bar_v, 0);
    tc_fence_after();
    if (vok) {
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)
        umma_bf16(tmem, kmaj_desc(sK, 128, ks), mnmaj_desc(sS, 128, ks),
                  make_idesc(128, 128, 0, 1), ks > 0);
      umma_commit(&bar_m[2]);
    } else {
      mbar_arrive(&bar_m[2]);
    }
  }
  __syncwarp();
  // ---- o = scale (2^{G_t} O_inter + O_intra)
  if (!mbar_wait(&bar_m[2], 0)) ok = false;
  tc_fence_after();
  const float eg = exp2f(gt);
  // per-warp staging for coalesced output stores (8 rows x 64 bytes per
  // instruction): the Q region, free once the MMAs above are done
  const uint32_t scratch = sQ + warp * 2048;
  const int t0 = j * 128 + quad * 32;  // first token row of this warp
  if (__all_sync(0xffffffffu, ok)) {
#pragma unroll 1
    for (int c = 0; c < 2; ++c) {
      const int col0 = half * 64 + 32 * c;
      float a[32], b[32];
      tmem_ld32x2(lane_tmem + 128 + col0, a, lane_tmem + col0, b);
#pragma unroll
      for (int i = 0; i < 32; ++i) a[i] = p.scale * (eg * a[i] + b[i]);
      if (p.o_mode == 1) {
        const int b_ = bh / p.H, h = bh % p.H;
        const int nvalid = p.T - t0;
        const uint32_t valid = nvalid >= 32 ? 0xffffffffu : (nvalid <= 0 ? 0u : (1u << nvalid) - 1u);
        warp_store_block_bf16(scratch, a,
                              p.out + ((size_t(b_) * p.T + t0) * p.H + h) * p.DV + dv0 + col0,
                              size_t(p.H) * p.DV, valid);
      } else {
        warp_store_block_bf16(scratch, a, p.out + (size_t(bh) * p.TP + t0) * 128 + col0, 128,
                              0xffffffffu);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// ============================================================ tile output with readout, 2 CTAs/SM
// Pass 1's output tile and the slot readout in about 97 KiB of shared memory,
// so that two CTAs share an SM and one CTA's loads and MMAs run during the
// other's epilogues.  Q, K and the state S_j stream
// through two 48 KiB stages in 64-wide k-blocks (Q | K | S rows of the block);
// the stages are then reused:
//   stage 0: V (32 KiB) once k-block NKB-2 is done, then z; table panel 0 at +32 KiB
//   stage 1: P once all k-blocks are done, then the store staging and p; table
//            panel 1 at +32 KiB
// TMEM (256 columns): [0,128) Q K^T -> P V -> logits;  [128,256) Q S_j -> p Tab.
constexpr int kRoStage = 49152;
constexpr int kRoSmem = 2 * kRoStage + 1024;

template <int DK>
__global__ void __launch_bounds__(256, 2)
    tile_fwd_ro_kernel(const __grid_constant__ CUtensorMap map_q,
                       const __grid_constant__ CUtensorMap map_k,
                       const __grid_constant__ CUtensorMap map_v,
                       const __grid_constant__ CUtensorMap map_s64,
                       const __grid_constant__ CUtensorMap map_tab, TileFwdParams p) {
  constexpr int NKB = DK / 64;
  static_assert(NKB % 2 == 0, "k-blocks alternate between the two stages");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  __shared__ __align__(8) uint64_t full[2], empty[2], bar_v, bar_tab[2], bar_m[4];
  __shared__ uint32_t tmem_base;
  __shared__ float Gs[128];
  __shared__ float xch[2][128];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, half = warp >> 2;
  const int r = quad * 32 + lane;
  const int bh = blockIdx.x / p.NT, j = blockIdx.x % p.NT;
  const int t = j * 128 + r;

  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(&bar_v, 1);
    mbar_init(&bar_tab[0], 1);
    mbar_init(&bar_tab[1], 1);
    for (int i = 0; i < 4; ++i) mbar_init(&bar_m[i], 1);
    mbar_fence_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base, 256);
    tmem_relinquish();  // one allocation per CTA: let the co-resident CTA allocate
  }
  pdl_wait();
  if (tid < 128) Gs[tid] = p.G[size_t(bh) * p.TP + j * 128 + tid];
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_trigger();
  const uint32_t tmem = tmem_base;
  const uint32_t lane_tmem = tmem + ((quad * 32) << 16);
  const uint32_t st0 = smem_u32(smem), st1 = st0 + kRoStage;
  const uint32_t tab0 = st0 + 32768, tab1 = st1 + 32768;
  bool ok = true;
  // copies issued by thread 0 (for the drain after a failed wait)
  int issued = 0, consumed = 0;
  bool v_issued = false, tab_issued[2] = {false, false};

  if (tid == 0) {
    // ---- Q K^T and Q S_j over the k-blocks
    auto issue = [&](int kb) {
      const int s = kb & 1;
      uint8_t* b = smem + s * kRoStage;
      mbar_expect_tx(&full[s], kRoStage);
      load_token_tile(b, &map_q, kRows2D, bh, p.H, p.TP, j, 64 * kb, 64, &full[s]);
      load_token_tile(b + 16384, &map_k, kRows2D, bh, p.H, p.TP, j, 64 * kb, 64, &full[s]);
      for (int c = 0; c < 2; ++c)
        tma_load_2d(b + 32768 + c * 8192, &map_s64, &full[s], 64 * c,
                    (bh * p.NT + j) * DK + 64 * kb);
      ++issued;
    };
    issue(0);
    issue(1);
    for (int kb = 0; kb < NKB && ok; ++kb) {
      const int s = kb & 1;
      if (!mbar_wait(&full[s], (kb >> 1) & 1)) {
        ok = false;
        break;
      }
      consumed = kb + 1;
      tc_fence_after();
      const uint32_t sq = s ? st1 : st0, sk = sq + 16384, ss = sq + 32768;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        umma_bf16(tmem, kmaj_desc(sq, 128, ks), kmaj_desc(sk, 128, ks), make_idesc(128, 128, 0, 0),
                  kb > 0 || ks > 0);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        umma_bf16(tmem + 128, kmaj_desc(sq, 128, ks), mnmaj_desc(ss, 64, ks),
                  make_idesc(128, 128, 0, 1), kb > 0 || ks > 0);
      umma_commit(&empty[s]);
      // the stage's next use once these MMAs are done: k-block kb + 2, or (the
      // last two k-blocks) V and table panel 0 into stage 0 / panel 1 into stage 1
      if (!mbar_wait(&empty[s], (kb >> 1) & 1)) {
        ok = false;
        break;
      }
      if (kb + 2 < NKB) {
        issue(kb + 2);
      } else if (s == 0) {
        mbar_expect_tx(&bar_v, 32768);
        load_token_tile(smem, &map_v, p.v_mode, bh, p.H, p.TP, j, 0, 128, &bar_v);
        v_issued = true;
        mbar_expect_tx(&bar_tab[0], 16384);
        tma_load_2d(smem + 32768, &map_tab, &bar_tab[0], 0, (bh % p.H) * 128);
        tab_issued[0] = true;
      } else {
        mbar_expect_tx(&bar_tab[1], 16384);
        tma_load_2d(smem + kRoStage + 32768, &map_tab, &bar_tab[1], 64, (bh % p.H) * 128);
        tab_issued[1] = true;
      }
    }
    umma_commit(&bar_m[0]);  // after the last k-block (or arrives at once on a failed wait)
  }
  const float gt = Gs[r];
  const float lam = p.lam[size_t(bh) * p.TP + t];
  __syncwarp();
  // ---- P = mask(S_qk o 2^{G_t - G_s}) -> bf16 K-major into stage 1
  if (!mbar_wait(&bar_m[0], 0)) ok = false;
  tc_fence_after();
  const uint32_t sP = st1;
  if (ok) {
#pragma unroll 1
    for (int c = 0; c < 2; ++c) {
      const int col0 = half * 64 + 32 * c;
      float v[32];
      tmem_ld32(lane_tmem + col0, v);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int s_ = col0 + i;
        v[i] = s_ <= r ? v[i] * exp2f(gt - Gs[s_]) : 0.f;
      }
      store_row32_bf16(sP + half * 16384, r, c * 4, v);
    }
  }
  fence_async_smem();
  tc_fence_before();
  ok = __syncthreads_and(ok);
  tc_fence_after();
  if (tid == 0) {
    ok = ok && mbar_wait(&bar_v, 0);
    if (ok) {
      tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)
        umma_bf16(tmem, kmaj_desc(sP, 128, ks), mnmaj_desc(st0, 128, ks),
                  make_idesc(128, 128, 0, 1), ks > 0);
      umma_commit(&bar_m[1]);
    } else {
      mbar_arrive(&bar_m[1]);
    }
  }
  __syncwarp();
  // ---- raw = scale (2^{G_t} O_inter + O_intra);  z = U(lam) bf16(raw) into stage 0
  if (!mbar_wait(&bar_m[1], 0)) ok = false;
  tc_fence_after();
  const float eg = exp2f(gt);
  const uint32_t scratch = st1 + warp * 2048;  // P is dead once P V is done
  const uint32_t sZ = st0;                     // V is dead once P V is done
  const int t0 = j * 128 + quad * 32;
  if (__all_sync(0xffffffffu, ok)) {
#pragma unroll 1
    for (int c = 0; c < 2; ++c) {
      const int col0 = half * 64 + 32 * c;
      float a[32], b[32];
      tmem_ld32x2(lane_tmem + 128 + col0, a, lane_tmem + col0, b);
#pragma unroll
      for (int i = 0; i < 32; ++i) a[i] = p.scale * (eg * a[i] + b[i]);
      warp_store_block_bf16(scratch, a, p.out + (size_t(bh) * p.TP + t0) * 128 + col0, 128,
                            0xffffffffu);
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        const float e = bf16_round(a[i]), o = bf16_round(a[i + 1]);
        float sn, cs;
        __sincosf(clock_phase(lam, col0 / 2 + i / 2), &sn, &cs);
        a[i] = cs * e - sn * o;
        a[i + 1] = sn * e + cs * o;
      }
      store_row32_bf16(sZ + half * 16384, r, c * 4, a);
    }
  }
  fence_async_smem();
  tc_fence_before();
  ok = __syncthreads_and(ok);
  tc_fence_after();
  if (tid == 0) {
    ok = ok && mbar_wait(&bar_tab[0], 0) && mbar_wait(&bar_tab[1], 0);
    if (ok) {
      tc_fence_after();
      // logits = z Tab^T: the table's two 64-column panels are a stage apart
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)
        umma_bf16(tmem, kmaj_desc(sZ, 128, ks),
                  make_sdesc((ks < 4 ? tab0 : tab1) + (ks & 3) * 32, 16, 1024),
                  make_idesc(128, 128, 0, 0), ks > 0);
      umma_commit(&bar_m[2]);
    } else {
      mbar_arrive(&bar_m[2]);
    }
  }
  __syncwarp();
  if (!mbar_wait(&bar_m[2], 0)) ok = false;
  tc_fence_after();
  // ---- softmax over the 127 active slots; each thread holds half of its token's row
  float l[64];
  tmem_ld32(lane_tmem + half * 64, *reinterpret_cast<float(*)[32]>(l));
  tmem_ld32(lane_tmem + half * 64 + 32, *reinterpret_cast<float(*)[32]>(l + 32));
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
#pragma unroll
  for (int i = 0; i < 64; ++i) l[i] *= inv;
  const uint32_t sPr = st1;  // the staging of the raw stores is done
  if (ok) store_row64_bf16(sPr + half * 16384, r, l);
  fence_async_smem();
  tc_fence_before();
  ok = __syncthreads_and(ok);
  tc_fence_after();
  if (tid == 0) {
    if (ok) {
      // p Tab: the table as an MN-major operand, 64-column blocks a stage apart
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)
        umma_bf16(tmem + 128, kmaj_desc(sPr, 128, ks), make_sdesc(tab0 + ks * 2048, kRoStage, 1024),
                  make_idesc(128, 128, 0, 1), ks > 0);
      umma_commit(&bar_m[3]);
    } else {
      mbar_arrive(&bar_m[3]);
    }
  }
  __syncwarp();
  if (!mbar_wait(&bar_m[3], 0)) ok = false;
  tc_fence_after();
  // ---- weights = U(-lam) (p Tab)
  if (__all_sync(0xffffffffu, ok)) {
#pragma unroll 1
    for (int c = 0; c < 2; ++c) {
      const int col0 = half * 64 + 32 * c;
      float v[32];
      tmem_ld32(lane_tmem + 128 + col0, v);
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        float sn, cs;
        __sincosf(clock_phase(lam, col0 / 2 + i / 2), &sn, &cs);
        const float e = v[i], o = v[i + 1];
        v[i] = cs * e + sn * o;
        v[i + 1] = -sn * e + cs * o;
      }
      // staging: p (stage 1) is dead once p Tab is done
      warp_store_block_bf16(scratch, v, p.weights + (size_t(bh) * p.TP + t0) * 128 + col0, 128,
                            0xffffffffu);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (tid == 0 && !ok) {
    // after a failed wait, copies may be in flight: let them land before exit
    for (int kb = consumed; kb < issued; ++kb) mbar_wait(&full[kb & 1], (kb >> 1) & 1);
    if (v_issued) mbar_wait(&bar_v, 0);
    for (int i = 0; i < 2; ++i)
      if (tab_issued[i]) mbar_wait(&bar_tab[i], 0);
  }
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

}  // namespace cyfa
