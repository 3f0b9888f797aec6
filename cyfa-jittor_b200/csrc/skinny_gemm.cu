// Weight-streaming GEMM for few rows: y[M, N] = x[M, K] W[N, K]^T with M <= 256,
// the shape of every projection of a batched decode step (M = sequences in the
// batch, W an nn.Linear weight).  At M = 256 a bf16 weight element feeds 2 x 256
// FLOPs, right at the B200's ridge (~255 FLOP/B), so the GEMM should run at the
// HBM rate of the weights; a library GEMM tuned for large M leaves most of the
// weight bytes idle (tiles of 64 x 64 that each walk all of K).
//
// Structure (one CTA of 192 threads per 128-column slice of W and K split s):
//   warp 0 (lane 0): TMA producer; per 64-wide k-block one [128 x 64] tile of W
//                    and one or two [128 x 64] tiles of x into a ring of stages;
//   warp 1 (lane 0): MMA issuer; per k-block 4 k16-steps of tcgen05.mma for
//                    each 128-row half of x, accumulating in TMEM (128 columns
//                    per half); a stage is released by tcgen05.commit;
//   warps 2-5      : epilogue; TMEM lane quadrant (warp % 4), 128 columns per
//                    row: bf16 y directly (one split) or fp32 partials that
//                    skinny_reduce_kernel sums in split order (deterministic).
// x comes from L2 after its first read (every CTA reads the same x rows);
// W is read from HBM exactly once.  All waits are bounded (mbar_wait, 2 s);
// on a timeout every role stops, copies in flight land, TMEM is freed.
#include "cyfa_common.cuh"

namespace cyfa {

struct SkinnyParams {
  int M, N, K;
  int S;                 // K splits
  __nv_bfloat16* y;      // [M, N] rows ldy apart (S == 1)
  long long ldy;
  float* part;           // [S, M, N] fp32 partials (S > 1)
};

constexpr int kSkinnyThreads = 192;

template <int MT>
struct SkinnyCfg {
  static constexpr int stages = MT == 2 ? 4 : 6;
  static constexpr int stage_bytes = (1 + MT) * 16384;  // W tile + MT x tiles
  static constexpr int smem = stages * stage_bytes + 1024;
};

template <int MT>
__global__ void __launch_bounds__(kSkinnyThreads, 1)
    skinny_gemm_kernel(const __grid_constant__ CUtensorMap map_x,
                       const __grid_constant__ CUtensorMap map_w, SkinnyParams p) {
  constexpr int STAGES = SkinnyCfg<MT>::stages;
  constexpr int STAGE = SkinnyCfg<MT>::stage_bytes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[STAGES], empty[STAGES], done;
  __shared__ uint32_t tmem_base;
  __shared__ int s_abort;
  volatile int* abort_flag = &s_abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * 128, split = blockIdx.y;
  const int nkb = p.K / 64;
  const int kb0 = int((long long)split * nkb / p.S), kb1 = int((long long)(split + 1) * nkb / p.S);
  const int nloc = kb1 - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&done, 1);
    s_abort = 0;
    mbar_fence_init();
    prefetch_tmap(&map_x);
    prefetch_tmap(&map_w);
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base, 128 * MT);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();
  pdl_trigger();
  const uint32_t tmem = tmem_base;

  if (warp == 0) {
    // ------------------------------------------------ producer
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < nloc; ++i) {
        if (*abort_flag) break;
        const int s = i % STAGES;
        if (i >= STAGES && !mbar_wait(&empty[s], ((i / STAGES) - 1) & 1)) {
          *abort_flag = 1;
          break;
        }
        uint8_t* st = smem + s * STAGE;
        const int k = (kb0 + i) * 64;
        mbar_expect_tx(&full[s], STAGE);
        tma_load_2d(st, &map_w, &full[s], k, n0);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) tma_load_2d(st + 16384 * (1 + mt), &map_x, &full[s], k, mt * 128);
        issued = i + 1;
      }
      // every issued copy lands before shared memory goes away
      for (int i = issued > STAGES ? issued - STAGES : 0; i < issued; ++i)
        mbar_wait(&full[i % STAGES], (i / STAGES) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = make_idesc(128, 128, 0, 0);
      int issued = 0;
      for (int i = 0; i < nloc; ++i) {
        const int s = i % STAGES;
        if (*abort_flag || !mbar_wait(&full[s], (i / STAGES) & 1)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t wb = smem_u32(smem + s * STAGE);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            umma_bf16(tmem + 128 * mt, kmaj_desc(wb + 16384 * (1 + mt), 128, ks),
                      kmaj_desc(wb, 128, ks), idesc, (i > 0 || ks > 0) ? 1u : 0u);
        }
        umma_commit(&empty[s]);
        issued = i + 1;
      }
      // `done` completes once every MMA issued above has finished (at once if
      // none was), so TMEM is not freed under a running MMA on the error path
      if (issued > 0) umma_commit(&done);
      else mbar_arrive(&done);
    }
  } else {
    // ------------------------------------------------ epilogue (warps 2-5)
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const bool got = mbar_wait(&done, 0) && *abort_flag == 0 && nloc > 0;
    tc_fence_after();
    if (got) {
#pragma unroll 1
      for (int mt = 0; mt < MT; ++mt) {
        const int m = mt * 128 + r;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          float v[32];
          tmem_ld32(tmem + 128 * mt + 32 * c + ((quad * 32) << 16), v);
          const int nb = n0 + 32 * c;
          if (m >= p.M || nb >= p.N) continue;
          if (p.S == 1) {
            __nv_bfloat16* dst = p.y + size_t(m) * p.ldy + nb;
#pragma unroll
            for (int e = 0; e < 32; e += 8)
              if (nb + e < p.N)
                *reinterpret_cast<uint4*>(dst + e) =
                    make_uint4(pack_bf16(v[e], v[e + 1]), pack_bf16(v[e + 2], v[e + 3]),
                               pack_bf16(v[e + 4], v[e + 5]), pack_bf16(v[e + 6], v[e + 7]));
          } else {
            float* dst = p.part + (size_t(split) * p.M + m) * p.N + nb;
#pragma unroll
            for (int e = 0; e < 32; e += 4)
              if (nb + e < p.N)
                *reinterpret_cast<float4*>(dst + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 128 * MT);
  }
}

// y[m, n] = bf16(sum_{s < S} part[s][m][n]), split order fixed; 8 columns per thread.
__global__ void __launch_bounds__(256) skinny_reduce_kernel(const float* part, int S, int M, int N,
                                                            __nv_bfloat16* y, long long ldy) {
  pdl_wait();
  pdl_trigger();
  const long long idx = (long long)blockIdx.x * 256 + threadIdx.x;
  const int per_row = N / 8;
  if (idx >= (long long)M * per_row) return;
  const int m = int(idx / per_row), n = int(idx % per_row) * 8;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int s = 0; s < S; ++s) {
    const float4* src = reinterpret_cast<const float4*>(part + (size_t(s) * M + m) * N + n);
    const float4 a = src[0], b = src[1];
    acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
    acc[4] += b.x; acc[5] += b.y; acc[6] += b.z; acc[7] += b.w;
  }
  *reinterpret_cast<uint4*>(y + size_t(m) * ldy + n) =
      make_uint4(pack_bf16(acc[0], acc[1]), pack_bf16(acc[2], acc[3]), pack_bf16(acc[4], acc[5]),
                 pack_bf16(acc[6], acc[7]));
}

// K splits: one CTA per 128-column slice when that fills at least half the SMs,
// else as many splits as fill the SMs once, at least 4 k-blocks each.
static int skinny_splits(int N, int K) {
  const int tiles = (N + 127) / 128, nkb = K / 64;
  if (tiles >= 74) return 1;
  int s = 148 / tiles;
  const int cap = nkb / 4 > 1 ? nkb / 4 : 1;
  if (s > cap) s = cap;
  return s < 1 ? 1 : s;
}

}  // namespace cyfa

using namespace cyfa;

extern "C" {

size_t cyfa_skinny_gemm_work_bytes(int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  const int S = skinny_splits(N, K);
  return S > 1 ? size_t(S) * M * N * sizeof(float) : 0;
}

int cyfa_skinny_gemm(const void* x, long long ldx, const void* w, void* y, long long ldy, int M,
                     int N, int K, void* work, size_t work_bytes, void* stream) {
  CYFA_REQUIRE(x && w && y, kNullPointer);
  CYFA_REQUIRE(M > 0 && M <= 256 && N > 0 && N % 8 == 0 && K > 0 && K % 64 == 0, kBadShape);
  CYFA_REQUIRE(ldx >= K && ldx % 8 == 0 && ldy >= N && ldy % 8 == 0, kBadShape);
  CYFA_REQUIRE(aligned(x, 16) && aligned(w, 16) && aligned(y, 16), kMisaligned);
  const int S = skinny_splits(N, K);
  const size_t need = cyfa_skinny_gemm_work_bytes(M, N, K);
  CYFA_REQUIRE(need == 0 || (work && work_bytes >= need && aligned(work, 16)), kWorkspace);
  CUtensorMap mx, mw;
  const uint64_t xd[2] = {uint64_t(K), uint64_t(M)};
  const uint64_t xs[1] = {uint64_t(ldx) * 2};
  const uint32_t box[2] = {64, 128};
  int rc = make_tmap_bf16(&mx, x, 2, xd, xs, box);
  if (rc) return rc;
  if ((rc = tmap_2d(&mw, w, uint64_t(N), uint64_t(K), 128))) return rc;
  SkinnyParams p{M, N, K, S, static_cast<__nv_bfloat16*>(y), ldy, static_cast<float*>(work)};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid((N + 127) / 128, S);
  if (M > 128) {
    set_smem(skinny_gemm_kernel<2>, SkinnyCfg<2>::smem);
    CYFA_LAUNCH("skinny_gemm", st, (launch_k(skinny_gemm_kernel<2>, grid, kSkinnyThreads,
                                             SkinnyCfg<2>::smem, st, mx, mw, p)));
  } else {
    set_smem(skinny_gemm_kernel<1>, SkinnyCfg<1>::smem);
    CYFA_LAUNCH("skinny_gemm", st, (launch_k(skinny_gemm_kernel<1>, grid, kSkinnyThreads,
                                             SkinnyCfg<1>::smem, st, mx, mw, p)));
  }
  rc = launch_status();
  if (rc || S == 1) return rc;
  const long long items = (long long)M * (N / 8);
  CYFA_LAUNCH("skinny_reduce", st,
              (launch_k(skinny_reduce_kernel, unsigned((items + 255) / 256), 256, 0, st,
                        static_cast<const float*>(work), S, M, N, static_cast<__nv_bfloat16*>(y),
                        ldy)));
  return launch_status();
}

}  // extern "C"
