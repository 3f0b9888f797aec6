// Output gate of the CyFA layer fused into its gated RMSNorm:
//   gate = gin Wg^T                          (the g_proj second linear, no bias)
//   y    = RMSNorm(scale * o) * w * sigmoid(gate + b)
// (reference layers/cyfa.py:350: o_norm(o * (num_slots - 1), g_proj(x)), with the
// g_proj second linear's bias added inside the sigmoid).  The gate linear is a
// K = head_v_dim contraction per (128-token tile, head): it runs on tcgen05 into
// TMEM and feeds the norm's epilogue directly, so the [tokens, H*D] gate tensor
// never goes to HBM (it is written only when the caller asks for it).
#include "cyfa_common.cuh"

namespace cyfa {

// sigmoid(z) = 1 / (1 + 2^(-z log2 e)) on the special-function unit: one ex2 and
// one reciprocal (relative error a few ulp; +-inf arguments give 0 and 1).
__device__ __forceinline__ float sigmoid_mufu(float z) {
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(z * -1.4426950408889634f));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.f + e));
  return r;
}

struct GateNormParams {
  int tokens, H, nk;           // nk = Kg / 64 k-blocks of the gate contraction
  float eps, scale;
  const float* w;              // [D] norm weight
  const __nv_bfloat16* gbias;  // [H*D] gate bias or null
  float* rstd;                 // [tokens*H]
  __nv_bfloat16* gate_out;     // [tokens, H*D] bf16 gate (pre-bias) or null
};

constexpr int kGnStages = 2;   // k-block ring: gin [128 x 64] + Wg_h [D x 64]
constexpr int kGnEpiWarps = 16;  // two groups of 8: group g finishes the units i with i % 2 == g
constexpr int kGnThreads = (kGnEpiWarps + 2) * 32;

template <int D>
constexpr int gn_stage_bytes() {
  return 128 * 128 + D * 128;
}
template <int D>
constexpr int gn_x_bytes() {
  return 128 * D * 2;
}
template <int D>
constexpr int gn_fwd_smem() {
  return kGnStages * gn_stage_bytes<D>() + 2 * gn_x_bytes<D>() + 1024;
}

// Persistent, warp-specialised; a unit is one (128-token tile, head), unit
// u -> tile u / H, head u % H, so the CTAs of one wave share their gin tiles
// through L2.  TMEM holds two D-column gate accumulators and shared memory two
// o tiles; the CTA's i-th unit uses buffer i % 2 of both.
//   warp 16, lane 0: TMA loads: per unit its nk k-blocks (gin tile columns,
//     the head's Wg rows) into the ring, then the o tile ([128, D] in D/64
//     swizzled column blocks) into its o buffer;
//   warp 17, lane 0: the k-block UMMAs (M = 128 tokens, N = D) into the unit's
//     TMEM buffer;
//   warps 0-15: epilogue in two groups of 8 warps, group g taking the units of
//     buffer g, so two units are finished side by side.  In a group, warp w
//     reads TMEM lane quadrant (w & 3) (token rows) and column half (w >> 2) & 1;
//     the row's sum of squares is joined from its two halves through shared
//     memory, then each thread writes y = n w sigmoid(bf16(gate) + b) over its
//     half of the o tile in shared memory, which one thread of the group stores
//     by TMA.
template <int D>
__global__ void __launch_bounds__(kGnThreads, 1)
    gate_norm_fwd_kernel(const __grid_constant__ CUtensorMap map_gin,
                         const __grid_constant__ CUtensorMap map_w,
                         const __grid_constant__ CUtensorMap map_x,
                         const __grid_constant__ CUtensorMap map_y, GateNormParams p) {
  constexpr int kStage = gn_stage_bytes<D>(), kX = gn_x_bytes<D>(), kHalf = D / 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* xbuf = smem + kGnStages * kStage;
  __shared__ __align__(8) uint64_t k_full[kGnStages], k_empty[kGnStages];
  __shared__ __align__(8) uint64_t x_full[2], x_empty[2], t_full[2], t_empty[2];
  __shared__ uint32_t tmem_base;
  __shared__ float ssx[2][128];  // per group: half-row sum of squares, then the row's rstd
  __shared__ int s_abort;
  volatile int* abort_flag = &s_abort;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int H = p.H, ntiles = (p.tokens + 127) / 128, nunits = ntiles * H;
  if (tid == 0) {
    for (int i = 0; i < kGnStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&x_full[i], 1);
      mbar_init(&x_empty[i], 1);
      mbar_init(&t_full[i], 1);
      mbar_init(&t_empty[i], 8);
    }
    s_abort = 0;
    mbar_fence_init();
    prefetch_tmap(&map_gin);
    prefetch_tmap(&map_w);
    prefetch_tmap(&map_x);
    prefetch_tmap(&map_y);
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base, 2 * D);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();
  pdl_trigger();
  const uint32_t tmem = tmem_base;

  if (warp == kGnEpiWarps) {
    // ------------------------------------------------ producer
    if (lane == 0) {
      int kq = 0, i = 0;
      for (int u = blockIdx.x; u < nunits && !*abort_flag; u += gridDim.x, ++i) {
        const int tile = u / H, h = u % H;
        bool ok = true;
        for (int c = 0; c < p.nk; ++c, ++kq) {
          const int s = kq % kGnStages;
          if (kq >= kGnStages && !mbar_wait(&k_empty[s], ((kq / kGnStages) - 1) & 1)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * kStage;
          mbar_expect_tx(&k_full[s], kStage);
          tma_load_2d(st, &map_gin, &k_full[s], 64 * c, tile * 128);
          tma_load_2d(st + 16384, &map_w, &k_full[s], 64 * c, h * D);
        }
        const int xs = i & 1;
        if (ok && i >= 2 && !mbar_wait(&x_empty[xs], ((i >> 1) - 1) & 1)) ok = false;
        if (!ok) {
          *abort_flag = 1;
          break;
        }
        mbar_expect_tx(&x_full[xs], kX);
#pragma unroll
        for (int cb = 0; cb < D / 64; ++cb)
          tma_load_3d(xbuf + xs * kX + cb * 16384, &map_x, &x_full[xs], 64 * cb, h, tile * 128);
      }
      // every issued copy lands before shared memory goes away
      for (int j = kq > kGnStages ? kq - kGnStages : 0; j < kq; ++j)
        mbar_wait(&k_full[j % kGnStages], (j / kGnStages) & 1);
      for (int j = i > 2 ? i - 2 : 0; j < i; ++j) mbar_wait(&x_full[j & 1], (j >> 1) & 1);
    }
  } else if (warp == kGnEpiWarps + 1) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = make_idesc(128, D, 0, 0);
      int kq = 0, i = 0;
      uint64_t* last_bar = nullptr;
      uint32_t last_par = 0;
      for (int u = blockIdx.x; u < nunits && !*abort_flag; u += gridDim.x, ++i) {
        const int b = i & 1;
        if (i >= 2 && !mbar_wait(&t_empty[b], ((i >> 1) - 1) & 1)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + b * D;
        bool ok = true;
        for (int c = 0; c < p.nk; ++c, ++kq) {
          const int s = kq % kGnStages;
          if (!mbar_wait(&k_full[s], (kq / kGnStages) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * kStage), sb = sa + 16384;
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            umma_bf16(acc, kmaj_desc(sa, 128, ks), kmaj_desc(sb, D, ks), idesc, c > 0 || ks > 0);
          umma_commit(&k_empty[s]);
          last_bar = &k_empty[s];
          last_par = (kq / kGnStages) & 1;
        }
        if (!ok) {
          *abort_flag = 1;
          break;
        }
        umma_commit(&t_full[b]);
        last_bar = &t_full[b];
        last_par = (i >> 1) & 1;
      }
      if (last_bar) mbar_wait(last_bar, last_par);  // all issued MMAs are done
    }
  } else {
    // ------------------------------------------------ epilogue
    const int grp = warp >> 3, quad = warp & 3, half = (warp >> 2) & 1;
    const int r = quad * 32 + lane;
    const uint32_t lane_tmem = tmem + ((quad * 32) << 16) + grp * D;
    const uint32_t xs = smem_u32(xbuf + grp * kX);
    const bool leader = (warp & 7) == 0 && lane == 0;
    const float scale2 = p.scale * p.scale;
    bool stores_pending = false;
    int n = 0;  // this group's units so far
    for (int u = blockIdx.x + grp * gridDim.x; u < nunits; u += 2 * gridDim.x, ++n) {
      const int tile = u / H, h = u % H;
      const int tok = tile * 128 + r;
      const bool got = __all_sync(0xffffffffu, *abort_flag == 0 &&
                                                   mbar_wait(&t_full[grp], n & 1) &&
                                                   mbar_wait(&x_full[grp], n & 1));
      // sum of squares of this thread's half row
      float ss0 = 0.f, ss1 = 0.f;
      if (got) {
#pragma unroll
        for (int q = 0; q < kHalf / 8; ++q) {
          float x[8];
          unpack_bf16x8(ld_shared_v4(xs + (half * (kHalf / 64) + (q >> 3)) * 16384 +
                                     sw128(r, q & 7)),
                        x);
#pragma unroll
          for (int e = 0; e < 8; e += 2) {
            ss0 = fmaf(x[e], x[e], ss0);
            ss1 = fmaf(x[e + 1], x[e + 1], ss1);
          }
        }
      }
      // join the halves through one float per row: half 0 posts its sum, half 1
      // adds its own and posts the row's rstd
      if (half == 0) ssx[grp][r] = ss0 + ss1;
      if (named_bar_or(1 + grp, 256, !got)) {
        *abort_flag = 1;
        break;
      }
      float rs;
      if (half == 1) {
        rs = rsqrtf((ssx[grp][r] + (ss0 + ss1)) * scale2 / D + p.eps);
        ssx[grp][r] = rs;
        if (tok < p.tokens) p.rstd[size_t(tok) * H + h] = rs;
      }
      named_bar_or(1 + grp, 256, false);
      if (half == 0) rs = ssx[grp][r];
      tc_fence_after();
      const float cr = p.scale * rs;
      const __nv_bfloat16* bias_h = p.gbias ? p.gbias + size_t(h) * D : nullptr;
#pragma unroll 1
      for (int cc = 0; cc < kHalf / 32; ++cc) {
        const int col = half * kHalf + 32 * cc;  // first of this step's 32 columns
        // the step's norm weights and gate biases (the same for every lane)
        float4 wq[8];
        uint4 bq[4];
#pragma unroll
        for (int k = 0; k < 8; ++k) wq[k] = __ldg(reinterpret_cast<const float4*>(p.w + col) + k);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          bq[k] = bias_h ? __ldg(reinterpret_cast<const uint4*>(bias_h + col) + k)
                         : make_uint4(0u, 0u, 0u, 0u);
        float g[32];
        tmem_ld32(lane_tmem + col, g);
        const uint32_t blk = xs + (col / 64) * 16384;
        const int q0 = (col % 64) / 8;
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
          const float wv[8] = {wq[2 * qq].x,     wq[2 * qq].y,     wq[2 * qq].z,
                               wq[2 * qq].w,     wq[2 * qq + 1].x, wq[2 * qq + 1].y,
                               wq[2 * qq + 1].z, wq[2 * qq + 1].w};
          float bias[8];
          unpack_bf16x8(bq[qq], bias);
          // the linear's output rounded to bf16, as a bf16 linear returns it
          const uint4 gq = make_uint4(pack_bf16(g[8 * qq + 0], g[8 * qq + 1]),
                                      pack_bf16(g[8 * qq + 2], g[8 * qq + 3]),
                                      pack_bf16(g[8 * qq + 4], g[8 * qq + 5]),
                                      pack_bf16(g[8 * qq + 6], g[8 * qq + 7]));
          float gt[8];
          unpack_bf16x8(gq, gt);
          const uint32_t addr = blk + sw128(r, q0 + qq);
          float x[8], y[8];
          unpack_bf16x8(ld_shared_v4(addr), x);
#pragma unroll
          for (int e = 0; e < 8; ++e) y[e] = (x[e] * cr) * (wv[e] * sigmoid_mufu(gt[e] + bias[e]));
          st_shared_v4(addr, pack_bf16(y[0], y[1]), pack_bf16(y[2], y[3]), pack_bf16(y[4], y[5]),
                       pack_bf16(y[6], y[7]));
          if (p.gate_out && tok < p.tokens)
            *reinterpret_cast<uint4*>(p.gate_out + (size_t(tok) * H + h) * D + col + 8 * qq) = gq;
        }
      }
      // hand the TMEM buffer back to the MMA issuer
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&t_empty[grp]);
      // y complete in shared memory: one thread stores it, then frees the buffer
      fence_async_smem();
      named_bar_or(1 + grp, 256, false);
      if (leader) {
#pragma unroll
        for (int cb = 0; cb < D / 64; ++cb)
          tma_store_3d(&map_y, xbuf + grp * kX + cb * 16384, 64 * cb, h, tile * 128);
        bulk_commit();
        bulk_wait_read_all();
        stores_pending = true;
        mbar_arrive(&x_empty[grp]);
      }
    }
    if (leader && stores_pending) bulk_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * D);
  }
}

}  // namespace cyfa

using namespace cyfa;

extern "C" {

int cyfa_gated_norm_gate_fwd(const void* x, const void* gin, long long gin_stride,
                             const void* gate_w, const void* gate_bias, int H, int Kg,
                             const float* w, float eps, float scale, void* y, float* rstd,
                             void* gate_out, int tokens, int D, void* stream) {
  CYFA_REQUIRE(x && gin && gate_w && w && y && rstd, kNullPointer);
  CYFA_REQUIRE(tokens > 0 && H > 0 && (D == 256 || D == 128) && Kg >= 64 && Kg % 64 == 0 &&
                   gin_stride >= Kg && gin_stride % 8 == 0,
               kBadShape);
  CYFA_REQUIRE(aligned(x, 16) && aligned(gin, 16) && aligned(gate_w, 16) && aligned(w, 16) &&
                   aligned(y, 16) && (!gate_bias || aligned(gate_bias, 16)) &&
                   (!gate_out || aligned(gate_out, 16)),
               kMisaligned);
  CUtensorMap mg, mw, mx, my;
  {
    const uint64_t dims[2] = {uint64_t(Kg), uint64_t(tokens)};
    const uint64_t strides[1] = {uint64_t(gin_stride) * 2};
    const uint32_t box[2] = {64, 128};
    int rc = make_tmap_bf16(&mg, gin, 2, dims, strides, box);
    if (rc) return rc;
  }
  {
    const uint64_t dims[2] = {uint64_t(Kg), uint64_t(H) * D};
    const uint64_t strides[1] = {uint64_t(Kg) * 2};
    const uint32_t box[2] = {64, uint32_t(D)};
    int rc = make_tmap_bf16(&mw, gate_w, 2, dims, strides, box);
    if (rc) return rc;
  }
  {
    const uint64_t dims[3] = {uint64_t(D), uint64_t(H), uint64_t(tokens)};
    const uint64_t strides[2] = {uint64_t(D) * 2, uint64_t(H) * D * 2};
    const uint32_t box[3] = {64, 1, 128};
    int rc = make_tmap_bf16(&mx, x, 3, dims, strides, box);
    if (rc) return rc;
    rc = make_tmap_bf16(&my, y, 3, dims, strides, box);
    if (rc) return rc;
  }
  GateNormParams p{tokens, H, Kg / 64, eps, scale, w,
                   static_cast<const __nv_bfloat16*>(gate_bias), rstd,
                   static_cast<__nv_bfloat16*>(gate_out)};
  const int nunits = ((tokens + 127) / 128) * H;
  const unsigned grid = unsigned(nunits < 148 ? nunits : 148);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (D == 256) {
    set_smem(gate_norm_fwd_kernel<256>, gn_fwd_smem<256>());
    CYFA_LAUNCH("gate_norm_fwd", s, (launch_k(gate_norm_fwd_kernel<256>, grid, kGnThreads,
                                              gn_fwd_smem<256>(), s, mg, mw, mx, my, p)));
  } else {
    set_smem(gate_norm_fwd_kernel<128>, gn_fwd_smem<128>());
    CYFA_LAUNCH("gate_norm_fwd", s, (launch_k(gate_norm_fwd_kernel<128>, grid, kGnThreads,
                                              gn_fwd_smem<128>(), s, mg, mw, mx, my, p)));
  }
  return launch_status();
}

}  // extern "C"
