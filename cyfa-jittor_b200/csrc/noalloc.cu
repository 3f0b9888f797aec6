// Allocation-free variant of the gated output-norm backward.
//
// cyfa_gated_norm_bwd needs a caller-provided work buffer for its per-block
// weight-gradient partial rows.  Some callers cannot provide one: bindings whose
// FFI signature carries only the op's own tensors (no workspace argument), and
// processes whose device memory is entirely owned by a framework allocator that
// does not let third-party libraries allocate.  For them,
// cyfa_gated_norm_bwd_static keeps the partial rows in a file-scope device array
// of fixed size instead, and calls no allocator.
//
// The array holds at most kStaticNormRows x 256 fp32 partials (296 KiB).  Every
// GPU that loads the library holds it until the process exits.  All calls share
// it: each call overwrites exactly the rows it later reads, so nothing needs to
// start at zero, but two calls whose kernels overlap on the GPU race on it.
#include <mutex>

#include "../../include/cyfa.h"
#include "cyfa_common.cuh"

namespace cyfa {

constexpr int kStaticNormRows = 296;  // = the largest block count of gated_norm_bwd
constexpr int kStaticNormCols = 256;  // largest supported head_v_dim
static __device__ __align__(256) float g_norm_scratch[kStaticNormRows * kStaticNormCols];

// Device address of g_norm_scratch on the current device.  In host code the
// array's name is only a host-side stand-in, so the address is looked up once
// per device (cudaGetSymbolAddress) and cached for the life of the process.  A
// device reset (cudaDeviceReset, or a reset of the primary context) reloads the
// module at a possibly different address, so the entry point is not for use on
// a device after such a reset.
static int static_norm_scratch(float** out) {
  static std::mutex mu;
  static float* cached[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return -static_cast<int>(e);
  if (dev < 0 || dev >= 64) return kBadShape;
  std::lock_guard<std::mutex> lk(mu);
  if (!cached[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_norm_scratch);
    if (e != cudaSuccess) return -static_cast<int>(e);
    cached[dev] = static_cast<float*>(p);
  }
  *out = cached[dev];
  return kOk;
}

}  // namespace cyfa

using namespace cyfa;

extern "C" {

int cyfa_gated_norm_bwd_static(const void* x, const void* gate, const float* w, float scale,
                               const float* rstd, const void* dy, void* dx, void* dgate,
                               float* dw, int rows, int D, void* stream) {
  CYFA_REQUIRE(aligned(w, 16), kMisaligned);
  CYFA_REQUIRE(x && gate && w && rstd && dy && dx && dgate && dw, kNullPointer);
  CYFA_REQUIRE(rows > 0 && (D == 256 || D == 128), kBadShape);
  const int nblk = norm_bwd_blocks(rows);
  // sizes beyond the fixed array are refused (cannot happen for D <= 256, checked anyway)
  CYFA_REQUIRE(nblk <= kStaticNormRows && size_t(nblk) * D <= size_t(kStaticNormRows) * kStaticNormCols,
               kWorkspace);
  float* part = nullptr;
  const int rc0 = static_norm_scratch(&part);
  if (rc0) return rc0;
  GatedNormParams p{static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(gate),
                    w, 0.f, scale, nullptr, const_cast<float*>(rstd),
                    static_cast<const __nv_bfloat16*>(dy), static_cast<__nv_bfloat16*>(dx),
                    static_cast<__nv_bfloat16*>(dgate), part, rows};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (D == 256)
    CYFA_LAUNCH("gated_norm_bwd", s, (launch_k(gated_norm_bwd_kernel<8>, nblk, 256, 0, s, p)));
  else
    CYFA_LAUNCH("gated_norm_bwd", s, (launch_k(gated_norm_bwd_kernel<4>, nblk, 256, 0, s, p)));
  int rc = launch_status();
  if (rc) return rc;
  CYFA_LAUNCH("column_sum", s,
              (launch_k(column_sum_kernel, (D + 31) / 32, 1024, 0, s, part, dw, nblk, D, nullptr,
                        nullptr, 0x7fffffff, nullptr)));
  return launch_status();
}

}  // extern "C"
