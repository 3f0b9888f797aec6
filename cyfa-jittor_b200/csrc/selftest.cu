// Self-test GEMM for the tcgen05 building blocks: C[128 x N] = A[128 x K] * B[K x N]
// with A and B staged by TMA (128-byte swizzle) in either K-major or MN-major
// form, accumulated in TMEM and read back with tcgen05.ld.  It exercises
// exactly the descriptor/swizzle encodings that the chunk kernels use, so a
// GPU test can compare it with a library matmul before trusting them.
#include "cyfa_common.cuh"

namespace cyfa {

struct SelftestParams {
  int K, N;        // K in {64,128,192,256}, N in {64,128,256}
  int a_mn, b_mn;  // operand majors
  float* c;        // [128, N] fp32
};

__global__ void __launch_bounds__(128) umma_selftest_kernel(
    const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
    SelftestParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sa = smem;                      // 128 * K * 2 bytes
  uint8_t* sb = smem + 128 * p.K * 2;      // N * K * 2 bytes
  __shared__ __align__(8) uint64_t bar_load, bar_mma;
  __shared__ uint32_t tmem_base;
  const int warp = threadIdx.x >> 5;

  if (threadIdx.x == 0) {
    mbar_init(&bar_load, 1);
    mbar_init(&bar_mma, 1);
    mbar_fence_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base, 256);
    tmem_relinquish();  // one allocation per CTA: let co-resident CTAs allocate
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  bool ok = true;

  if (threadIdx.x == 0) {
    const uint32_t bytes = (128 + p.N) * p.K * 2;
    mbar_expect_tx(&bar_load, bytes);
    // A: K-major -> blocks of [128 rows x 64 k]; MN-major -> blocks of [K rows x 64 m].
    if (!p.a_mn) {
      for (int kb = 0; kb < p.K / 64; ++kb) tma_load_2d(sa + kb * 128 * 128, &tma_a, &bar_load, kb * 64, 0);
    } else {
      for (int mb = 0; mb < 2; ++mb) tma_load_2d(sa + mb * p.K * 128, &tma_a, &bar_load, mb * 64, 0);
    }
    if (!p.b_mn) {
      for (int kb = 0; kb < p.K / 64; ++kb) tma_load_2d(sb + kb * p.N * 128, &tma_b, &bar_load, kb * 64, 0);
    } else {
      for (int nb = 0; nb < p.N / 64; ++nb) tma_load_2d(sb + nb * p.K * 128, &tma_b, &bar_load, nb * 64, 0);
    }
    ok = mbar_wait(&bar_load, 0);
    tc_fence_after();
    if (ok) {
      const uint32_t idesc = make_idesc(128, p.N, p.a_mn, p.b_mn);
      const uint32_t a0 = smem_u32(sa), b0 = smem_u32(sb);
      for (int ks = 0; ks < p.K / 16; ++ks) {
        uint64_t ad, bd;
        if (!p.a_mn)
          ad = make_sdesc(a0 + (ks >> 2) * 128 * 128 + (ks & 3) * 32, 16, 1024);
        else
          ad = make_sdesc(a0 + ks * 2048, p.K * 128, 1024);
        if (!p.b_mn)
          bd = make_sdesc(b0 + (ks >> 2) * p.N * 128 + (ks & 3) * 32, 16, 1024);
        else
          bd = make_sdesc(b0 + ks * 2048, p.K * 128, 1024);
        umma_bf16(tmem, ad, bd, idesc, ks > 0);
      }
      umma_commit(&bar_mma);
    } else {
      mbar_arrive(&bar_mma);
    }
  }
  __syncwarp();
  ok = mbar_wait(&bar_mma, 0);
  tc_fence_after();
  if (ok) {
    const int row = threadIdx.x;
    const uint32_t lane_addr = tmem_lane_base(tmem);
    for (int c0 = 0; c0 < p.N; c0 += 32) {
      float v[32];
      tmem_ld32(lane_addr + c0, v);
      for (int i = 0; i < 32; ++i) p.c[row * p.N + c0 + i] = v[i];
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

}  // namespace cyfa
