// Shared device helpers for the CyFA sm_100a kernels: mbarriers with
// time-bounded waits, TMA tile loads, tcgen05 (UMMA + TMEM) wrappers,
// shared-memory matrix descriptors and the 128-byte swizzle address map.
//
// Every wait in this library is bounded by wall-clock time (%globaltimer).
// When a wait runs out the kernel records an error code in the device-side
// error word (read back through cyfa_device_error()) and unwinds: it stops
// issuing work, waits (again bounded) for its own in-flight copies, frees its
// TMEM and returns.  Nothing here traps or spins without a limit.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#ifndef CYFA_WAIT_NS
#define CYFA_WAIT_NS 2000000000ull  // 2 s per wait before giving up
#endif

namespace cyfa {

// Device error word: 0 = ok; otherwise the first failing site's code.  The
// library is built as one translation unit (cyfa_all.cu), so this is its only
// definition.
__device__ int g_device_error = 0;

enum DeviceError : int {
  kErrNone = 0,
  kErrWaitTimeout = 1,
  kErrBadShape = 2,
};

__device__ __forceinline__ void set_error(int code) { atomicCAS(&g_device_error, 0, code); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Programmatic dependent launch.  Every kernel of this library calls pdl_wait()
// before its first global-memory access (it returns once the grids this launch
// depends on have completed and their writes are visible; without a
// programmatic dependency it returns at once) and pdl_trigger() once it holds
// its on-chip resources (after any TMEM allocation), which lets the next
// kernel in the stream launch and run its own prologue early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Waits for the phase with the given parity to complete; false on timeout
// (the error word is set).  Callers must unwind on false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - start > CYFA_WAIT_NS) {
      set_error(kErrWaitTimeout);
      return false;
    }
  }
}

// ---------------------------------------------------------------- TMA
// Tiled tensor loads (no multicast), completion signalled on an mbarrier.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, uint64_t* bar, int x,
                                            int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, uint64_t* bar, int x,
                                            int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void tma_load_4d(void* dst, const void* tmap, uint64_t* bar, int x,
                                            int y, int z, int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}
// Tiled tensor store from shared memory (bulk async group of the issuing
// thread).  Rows or columns outside the tensor are not written.
__device__ __forceinline__ void tma_store_3d(const void* tmap, const void* src, int x, int y,
                                             int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          tmap),
      "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Waits until the committed bulk stores of this thread have read their shared
// memory sources (the buffers may be reused), or until they are complete.
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
// Coalesced warp load of a 32-row x 32-column bf16 block (the inverse of
// warp_store_block_bf16, in two steps so that the global loads can be issued
// early): warp_fetch_block_bf16 reads 8 rows x 64 contiguous bytes per
// instruction into `raw` (lane l holds row 8k + l/4, 16-byte chunk l%4, k = 0..3);
// warp_transpose_block_bf16 passes them through the warp's 2 KiB staging buffer
// and returns row `lane` (32 values as 4 x 8 bf16).
__device__ __forceinline__ void warp_fetch_block_bf16(const __nv_bfloat16* src, size_t stride,
                                                      uint4 (&raw)[4]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < 4; ++k)
    raw[k] = *reinterpret_cast<const uint4*>(src + (8 * k + (lane >> 2)) * stride + (lane & 3) * 8);
}
// Plain bulk copy of `bytes` contiguous bytes (16-byte aligned, a multiple of
// 16) from global to shared memory; completion on an mbarrier.  No multicast.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// Ampere-style asynchronous 16-byte copies (zero fill when `valid` is false).
__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* gsrc, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(saddr), "l"(gsrc),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Generic-proxy smem writes must be fenced before the async proxy (UMMA) reads.
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem], kind::f16 (bf16 in, fp32 accumulate), one CTA.
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
// Arrives once on the mbarrier when all previously issued MMAs of this thread finish.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// Instruction descriptor: bf16 x bf16 -> fp32, M x N tile, operand majors
// (0 = K-major, 1 = MN-major).
__host__ __device__ constexpr uint32_t make_idesc(int M, int N, int a_mn, int b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(a_mn) << 15) | (uint32_t(b_mn) << 16) |
         (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}

// Shared-memory matrix descriptor, 128-byte swizzle, sm100 version bit.
// K-major: rows of 128 B (64 bf16 of K), 8-row groups at sbo (1024 when dense).
// MN-major: 128 B holds 64 MN elements, K rows at 128 B, 8-row groups at sbo,
// 64-element MN blocks at lbo.
__device__ __forceinline__ uint64_t make_sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return uint64_t((saddr >> 4) & 0x3FFF) | (uint64_t((lbo >> 4) & 0x3FFF) << 16) |
         (uint64_t((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46) | (2ull << 61);
}

// TMEM -> registers: 32 lanes x 32 consecutive fp32 columns per warp.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// TMEM lane base of this warp's 32-lane sub-partition.
__device__ __forceinline__ uint32_t tmem_lane_base(uint32_t tmem) {
  return tmem + (((threadIdx.x >> 5) & 3u) * 32u << 16);
}

// ---------------------------------------------------------------- swizzle
// Byte offset of (row, 16-byte chunk) inside a 128B-swizzled block whose rows
// are 128 bytes wide.  Block bases must be 1024-byte aligned.
__device__ __forceinline__ uint32_t sw128(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

// Writes 64 consecutive fp32 values of one row (this thread's row) as bf16 into
// a K-major (or MN-major: same bytes) 128B-swizzled operand block: `block` is
// the 1024-aligned base of the [rows x 64] block.
__device__ __forceinline__ void store_row64_bf16(uint32_t block, uint32_t row, const float* v) {
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    st_shared_v4(block + sw128(row, c), pack_bf16(v[8 * c + 0], v[8 * c + 1]),
                 pack_bf16(v[8 * c + 2], v[8 * c + 3]), pack_bf16(v[8 * c + 4], v[8 * c + 5]),
                 pack_bf16(v[8 * c + 6], v[8 * c + 7]));
  }
}

// Writes 32 consecutive values (half a 64-wide block row) starting at chunk c0.
__device__ __forceinline__ void store_row32_bf16(uint32_t block, uint32_t row, int c0,
                                                 const float* v) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    st_shared_v4(block + sw128(row, c0 + c), pack_bf16(v[8 * c + 0], v[8 * c + 1]),
                 pack_bf16(v[8 * c + 2], v[8 * c + 3]), pack_bf16(v[8 * c + 4], v[8 * c + 5]),
                 pack_bf16(v[8 * c + 6], v[8 * c + 7]));
  }
}

// Operand descriptors of a tile stored as 64-column blocks of [R x 64]
// (one 128-byte swizzled row per tile row), for MMA k-step ks (16 elements).
// K-major operand: R rows of the M (or N) dimension, K along the columns.
__device__ __forceinline__ uint64_t kmaj_desc(uint32_t base, int R, int ks) {
  return make_sdesc(base + (ks >> 2) * R * 128 + (ks & 3) * 32, 16, 1024);
}
// MN-major operand: R rows of the K dimension, M (or N) along the columns.
__device__ __forceinline__ uint64_t mnmaj_desc(uint32_t base, int R, int ks) {
  return make_sdesc(base + ks * 2048, R * 128, 1024);
}

// Loads 16 bytes (8 bf16) of row `row`, chunk c of a swizzled block.
__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

// Two 32-column TMEM loads with one completion wait.
#define CYFA_TMEM_LD32_ASM(dst, taddr)                                                          \
  asm volatile(                                                                                  \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"   \
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"         \
      : "=r"(dst[0]), "=r"(dst[1]), "=r"(dst[2]), "=r"(dst[3]), "=r"(dst[4]), "=r"(dst[5]),     \
        "=r"(dst[6]), "=r"(dst[7]), "=r"(dst[8]), "=r"(dst[9]), "=r"(dst[10]), "=r"(dst[11]),   \
        "=r"(dst[12]), "=r"(dst[13]), "=r"(dst[14]), "=r"(dst[15]), "=r"(dst[16]),             \
        "=r"(dst[17]), "=r"(dst[18]), "=r"(dst[19]), "=r"(dst[20]), "=r"(dst[21]),             \
        "=r"(dst[22]), "=r"(dst[23]), "=r"(dst[24]), "=r"(dst[25]), "=r"(dst[26]),             \
        "=r"(dst[27]), "=r"(dst[28]), "=r"(dst[29]), "=r"(dst[30]), "=r"(dst[31])              \
      : "r"(taddr))

__device__ __forceinline__ void tmem_ld32x2(uint32_t ta, float (&a)[32], uint32_t tb,
                                            float (&b)[32]) {
  uint32_t ra[32], rb[32];
  CYFA_TMEM_LD32_ASM(ra, ta);
  CYFA_TMEM_LD32_ASM(rb, tb);
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    a[i] = __uint_as_float(ra[i]);
    b[i] = __uint_as_float(rb[i]);
  }
}

__device__ __forceinline__ void warp_transpose_block_bf16(uint32_t scratch, const uint4 (&raw)[4],
                                                          uint4 (&row)[4]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int r = 8 * k + (lane >> 2), c = lane & 3;
    st_shared_v4(scratch + r * 64 + ((c ^ ((r >> 1) & 3)) << 4), raw[k].x, raw[k].y, raw[k].z,
                 raw[k].w);
  }
  __syncwarp();
#pragma unroll
  for (int c = 0; c < 4; ++c) row[c] = ld_shared_v4(scratch + lane * 64 + ((c ^ ((lane >> 1) & 3)) << 4));
  __syncwarp();
}

// The same for 32-row x 64-column bf16 blocks (128 bytes per row), staging
// buffer 4 KiB: lane l holds row l as 8 x 16-byte chunks; each global access
// instruction covers 4 rows x 128 contiguous bytes (lane l: row 4k + l/8, chunk l%8).
__device__ __forceinline__ void warp_store_rows128(uint32_t scratch, const uint4 (&row)[8],
                                                   __nv_bfloat16* dst, size_t stride) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int c = 0; c < 8; ++c)
    st_shared_v4(scratch + lane * 128 + ((c ^ (lane & 7)) << 4), row[c].x, row[c].y, row[c].z,
                 row[c].w);
  __syncwarp();
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int r = 4 * k + (lane >> 3), c = lane & 7;
    *reinterpret_cast<uint4*>(dst + r * stride + c * 8) =
        ld_shared_v4(scratch + r * 128 + ((c ^ (r & 7)) << 4));
  }
  __syncwarp();
}
__device__ __forceinline__ void warp_fetch_rows128(const __nv_bfloat16* src, size_t stride,
                                                   uint4 (&raw)[8]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < 8; ++k)
    raw[k] = *reinterpret_cast<const uint4*>(src + (4 * k + (lane >> 3)) * stride + (lane & 7) * 8);
}
__device__ __forceinline__ void warp_transpose_rows128(uint32_t scratch, const uint4 (&raw)[8],
                                                       uint4 (&row)[8]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int r = 4 * k + (lane >> 3), c = lane & 7;
    st_shared_v4(scratch + r * 128 + ((c ^ (r & 7)) << 4), raw[k].x, raw[k].y, raw[k].z, raw[k].w);
  }
  __syncwarp();
#pragma unroll
  for (int c = 0; c < 8; ++c) row[c] = ld_shared_v4(scratch + lane * 128 + ((c ^ (lane & 7)) << 4));
  __syncwarp();
}

// 2^x on the special-function unit (relative error about 2^-22; results below
// 2^-126 flush to zero).  Used for decay factors 2^{G_t - G_s} <= 1.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Warp-cooperative store of a 32-row x 32-column bf16 block.  Lane l holds the
// 32 values of row l (fp32); they are packed into the warp's 2 KiB staging
// buffer `scratch` (16-byte chunks XOR-swizzled, conflict-free both ways) and
// written back so that each store instruction covers 8 rows x 64 contiguous
// bytes instead of 32 rows x 16 bytes.  Row r goes to dst + r * stride
// (elements) when bit r of `valid` is set.
__device__ __forceinline__ void warp_store_block_bf16(uint32_t scratch, const float* v,
                                                      __nv_bfloat16* dst, size_t stride,
                                                      uint32_t valid) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int c = 0; c < 4; ++c)
    st_shared_v4(scratch + lane * 64 + ((c ^ ((lane >> 1) & 3)) << 4),
                 pack_bf16(v[8 * c], v[8 * c + 1]), pack_bf16(v[8 * c + 2], v[8 * c + 3]),
                 pack_bf16(v[8 * c + 4], v[8 * c + 5]), pack_bf16(v[8 * c + 6], v[8 * c + 7]));
  __syncwarp();
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int r = 8 * k + (lane >> 2), c = lane & 3;
    const uint4 val = ld_shared_v4(scratch + r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
    if ((valid >> r) & 1u) *reinterpret_cast<uint4*>(dst + r * stride + c * 8) = val;
  }
  __syncwarp();
}

__device__ __forceinline__ void unpack_bf16x8(const uint4& u, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 x = __bfloat1622float2(h[i]);
    f[2 * i] = x.x;
    f[2 * i + 1] = x.y;
  }
}

__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

}  // namespace cyfa
