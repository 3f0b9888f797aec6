// C-ABI entry points (include/cyfa.h): host-side argument checks, TMA tensor
// map construction and kernel launches.  No entry point allocates memory.
#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>
#include <set>
#include <tuple>
#include <vector>

#include "../../include/cyfa.h"
#include "cyfa_common.cuh"

namespace cyfa {

// Raises a kernel's dynamic shared memory limit once per (kernel, device); the
// attribute call is host-side only, so launches inside stream capture stay cheap.
template <typename Kern>
static void set_smem(Kern k, int bytes) {
  static std::mutex mu;
  static std::set<std::tuple<const void*, int, int>> done;
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_tuple(reinterpret_cast<const void*>(k), dev, bytes);
  std::lock_guard<std::mutex> lk(mu);
  if (done.count(key)) return;
  // the largest shared-memory carveout, so that kernels sized for two CTAs per SM
  // get them (the default carveout may leave room for one)
  cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout,
                       cudaSharedmemCarveoutMaxShared);
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) == cudaSuccess)
    done.insert(key);
}

enum Status : int {
  kOk = 0,
  kBadShape = 1,
  kNullPointer = 2,
  kMisaligned = 3,
  kBadDtype = 4,
  kNoDriver = 5,
  kTensorMap = 6,
  kWorkspace = 7,
};

#define CYFA_REQUIRE(cond, code) \
  do {                           \
    if (!(cond)) return (code);  \
  } while (0)

static int launch_status() {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? kOk : -static_cast<int>(e);
}

// Launch accounting and optional per-kernel timing.  Every kernel launch of the
// library goes through CYFA_LAUNCH, which counts it and, while profiling is on,
// brackets it with CUDA events on its own stream.
static std::atomic<long long> g_launches{0};
struct ProfRecord {
  const char* name;
  cudaEvent_t start, stop;
};
static std::mutex g_prof_mu;
static std::vector<ProfRecord> g_prof;
static bool g_prof_on = false;

static cudaEvent_t prof_begin(cudaStream_t s) {
  if (!g_prof_on) return nullptr;
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  cudaEventRecord(e, s);
  return e;
}
static void prof_end(const char* name, cudaEvent_t start, cudaStream_t s) {
  if (!start) return;
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  cudaEventRecord(e, s);
  std::lock_guard<std::mutex> lk(g_prof_mu);
  g_prof.push_back({name, start, e});
}

#define CYFA_LAUNCH(name, stream, ...)                 \
  do {                                                 \
    cudaEvent_t _cyfa_ev = prof_begin(stream);         \
    __VA_ARGS__;                                       \
    prof_end(name, _cyfa_ev, stream);                  \
    g_launches.fetch_add(1, std::memory_order_relaxed); \
  } while (0)

// Kernel launch with programmatic stream serialisation: the kernel may start
// while the previous kernel on the stream finishes (each kernel of this library
// waits in pdl_wait() before touching global memory), so launch latency and the
// prologue (barrier setup, TMEM allocation) overlap the previous kernel's tail.
// cyfa_set_pdl(0) turns it off (plain stream order).
static std::atomic<int> g_pdl{1};
// Segmented state scans for scans with fewer CTAs than SMs (cyfa_set_scan_split).
static std::atomic<int> g_scan_split{1};

template <typename... KArgs, typename... Args>
static void launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                     cudaStream_t stream, Args&&... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = g_pdl.load(std::memory_order_relaxed);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Auxiliary stream of the calling thread (cyfa_set_aux_stream).  A launch
// whose result no later kernel of the same entry point reads (a reduction into
// parameter gradients) goes to it when set, ordered after the work so far on
// the caller's stream; the caller makes its stream wait for the auxiliary one
// before the results are read.
static thread_local cudaStream_t t_aux = nullptr;

static cudaStream_t defer_stream(cudaStream_t st) {
  if (t_aux == nullptr || t_aux == st) return st;
  cudaEvent_t ev;
  if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) return st;
  const bool ok = cudaEventRecord(ev, st) == cudaSuccess &&
                  cudaStreamWaitEvent(t_aux, ev, 0) == cudaSuccess;
  cudaEventDestroy(ev);
  return ok ? t_aux : st;
}

static bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// cuTensorMapEncodeTiled through the runtime's driver entry point, so the
// library does not link libcuda directly.
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// bf16 tensor map, by default with a 128-byte swizzle and a box whose inner
// extent is 64 elements (one 128-byte row).  dims innermost first; strides in bytes for
// dims 1..rank-1.  Out-of-bounds elements are filled with zeros.
static int make_tmap_bf16(CUtensorMap* m, const void* base, int rank, const uint64_t* dims,
                          const uint64_t* strides, const uint32_t* box,
                          CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto fn = encode_fn();
  if (!fn) return kNoDriver;
  if (!aligned(base, 16)) return kMisaligned;
  for (int i = 0; i + 1 < rank; ++i)
    if (strides[i] % 16) return kMisaligned;
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) s[i] = strides[i];
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), d, s,
                        b, e, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? kOk : kTensorMap;
}

// 2-D row-major [rows, cols] bf16 matrix, box {64, box_rows}.
static int tmap_2d(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols,
                   uint32_t box_rows) {
  const uint64_t dims[2] = {cols, rows};
  const uint64_t strides[1] = {cols * 2};
  const uint32_t box[2] = {64, box_rows};
  return make_tmap_bf16(m, base, 2, dims, strides, box);
}

// Public-layout [B, T, H, K] bf16 rows `stride` elements apart as the 3-D map
// {H*K, T, B} with an unswizzled {K, 32, 1} box (one head's 32-token tile).
static int token_tmap(CUtensorMap* m, const void* base, int B, int T, int H, int K,
                      long long stride) {
  const uint64_t dims[3] = {uint64_t(H) * K, uint64_t(T), uint64_t(B)};
  const uint64_t strides[2] = {uint64_t(stride) * 2, uint64_t(stride) * 2 * uint64_t(T)};
  const uint32_t box[3] = {uint32_t(K), 32, 1};
  return make_tmap_bf16(m, base, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
}

}  // namespace cyfa

using namespace cyfa;

namespace cyfa {
static int token_fwd_launch(const void* q, const void* k, const float* q_norm_weight,
                            const float* k_norm_weight, const float* lam, const float* beta_h,
                            void* qn, void* kn, void* w, float* q_rs, float* k_rs, int B, int T,
                            int H, int K, float q_eps, float k_eps, long long q_stride,
                            long long k_stride, void* stream) {
  CYFA_REQUIRE(q && k && q_norm_weight && k_norm_weight && lam && beta_h && qn && kn && w &&
                   q_rs && k_rs,
               kNullPointer);
  CYFA_REQUIRE(B > 0 && T > 0 && H > 0 && (K == 128 || K == 256), kBadShape);
  CYFA_REQUIRE(aligned(q, 16) && aligned(k, 16) && q_stride % 8 == 0 && k_stride % 8 == 0 &&
                   aligned(qn, 16) && aligned(kn, 16) && aligned(w, 16) &&
                   aligned(q_norm_weight, 16) && aligned(k_norm_weight, 16),
               kMisaligned);
  const int TP = (T + 127) / 128 * 128;
  TokenFwdParams p{static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
                   q_norm_weight, k_norm_weight, lam, beta_h,
                   static_cast<__nv_bfloat16*>(qn), static_cast<__nv_bfloat16*>(kn),
                   static_cast<__nv_bfloat16*>(w), q_rs, k_rs, B, T, H, TP, q_eps, k_eps,
                   q_stride, k_stride};
  const size_t rows = size_t(B) * H * TP;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CUtensorMap mq, mk;
  if (token_tmap(&mq, q, B, T, H, K, q_stride) == kOk &&
      token_tmap(&mk, k, B, T, H, K, k_stride) == kOk) {
    const int ntiles = B * H * (TP / kTfRows);
    const unsigned grid = unsigned(ntiles < 296 ? ntiles : 296);  // persistent, two per SM
    if (K == 256) {
      set_smem(token_fwd_tma_kernel<256>, token_fwd_tma_smem<256>());
      CYFA_LAUNCH("token_fwd", s, launch_k(token_fwd_tma_kernel<256>, grid, 288,
                                           token_fwd_tma_smem<256>(), s, mq, mk, p));
    } else {
      set_smem(token_fwd_tma_kernel<128>, token_fwd_tma_smem<128>());
      CYFA_LAUNCH("token_fwd", s, launch_k(token_fwd_tma_kernel<128>, grid, 288,
                                           token_fwd_tma_smem<128>(), s, mq, mk, p));
    }
    return launch_status();
  }
  const dim3 grid(unsigned(token_fwd_blocks(rows)));
  if (K == 256) CYFA_LAUNCH("token_fwd", s, launch_k(token_fwd_kernel<256>, grid, 256, 0, s, p));
  else CYFA_LAUNCH("token_fwd", s, launch_k(token_fwd_kernel<128>, grid, 256, 0, s, p));
  return launch_status();
}

static int token_bwd_launch(const void* q, const void* k, const float* q_norm_weight,
                            const float* k_norm_weight, const float* q_rs, const float* k_rs,
                            const void* dqn, const void* dkn, const float* lam,
                            const float* beta_h, const void* dw, const void* dw_b, void* dq,
                            void* dk, float* dqw_part, float* dkw_part, float* dlam,
                            float* dbeta_h, int B,
                            int T, int H, int K, long long q_stride, long long k_stride,
                            long long dq_stride, long long dk_stride, bool grads_bf16,
                            void* stream, int* nblk_out = nullptr) {
  CYFA_REQUIRE(q && k && q_norm_weight && k_norm_weight && q_rs && k_rs && dqn && dkn && lam &&
                   beta_h && dw && dq && dk && dqw_part && dkw_part && dlam && dbeta_h,
               kNullPointer);
  CYFA_REQUIRE(B > 0 && T > 0 && H > 0 && (K == 128 || K == 256), kBadShape);
  CYFA_REQUIRE(aligned(q, 16) && aligned(k, 16) && aligned(dq, 16) && aligned(dk, 16) &&
                   aligned(dqn, 16) && aligned(dkn, 16) && aligned(dw, 16) &&
                   (!dw_b || aligned(dw_b, 16)) && aligned(q_norm_weight, 16) &&
                   aligned(k_norm_weight, 16) && q_stride % 8 == 0 && k_stride % 8 == 0 &&
                   dq_stride % 8 == 0 && dk_stride % 8 == 0,
               kMisaligned);
  const int TP = (T + 127) / 128 * 128;
  TokenBwdParams p{static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
                   q_norm_weight, k_norm_weight, q_rs, k_rs, dqn, dkn, lam, beta_h, dw, dw_b,
                   static_cast<__nv_bfloat16*>(dq), static_cast<__nv_bfloat16*>(dk), dqw_part,
                   dkw_part, dlam, dbeta_h, B, T, H, TP, q_stride, k_stride, dq_stride,
                   dk_stride};
  const size_t rows = size_t(B) * H * TP;
  const dim3 grid(unsigned(token_bwd_blocks(rows)));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // with bf16 gradients, for a caller that takes the partial-row count: the
  // TMA-streamed kernel (one partial row per persistent CTA)
  CUtensorMap mq, mk, mdq, mdk, mdw, mdwb;
  auto map2 = [&](CUtensorMap* m, const void* base, int cols) {
    const uint64_t dims[2] = {uint64_t(cols), uint64_t(rows)};
    const uint64_t strides[1] = {uint64_t(cols) * 2};
    const uint32_t box[2] = {uint32_t(cols), 32};
    return make_tmap_bf16(m, base, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
  };
  if (grads_bf16 && nblk_out && token_tmap(&mq, q, B, T, H, K, q_stride) == kOk &&
      token_tmap(&mk, k, B, T, H, K, k_stride) == kOk && map2(&mdq, dqn, K) == kOk &&
      map2(&mdk, dkn, K) == kOk && map2(&mdw, dw, 128) == kOk &&
      (!dw_b || map2(&mdwb, dw_b, 128) == kOk)) {
    if (!dw_b) mdwb = mdw;
    const int ntiles = B * H * (TP / kTbRows);
    const unsigned g = unsigned(ntiles < 148 ? ntiles : 148);  // persistent
    if (K == 256) {
      set_smem(token_bwd_tma_kernel<256>, token_bwd_tma_smem<256>());
      CYFA_LAUNCH("token_bwd", s, (launch_k(token_bwd_tma_kernel<256>, g, 288,
                                            token_bwd_tma_smem<256>(), s, mq, mk, mdq, mdk, mdw,
                                            mdwb, p)));
    } else {
      set_smem(token_bwd_tma_kernel<128>, token_bwd_tma_smem<128>());
      CYFA_LAUNCH("token_bwd", s, (launch_k(token_bwd_tma_kernel<128>, g, 288,
                                            token_bwd_tma_smem<128>(), s, mq, mk, mdq, mdk, mdw,
                                            mdwb, p)));
    }
    *nblk_out = int(g);
    return launch_status();
  }
  if (nblk_out) *nblk_out = int(grid.x);
  if (grads_bf16) {
    if (K == 256)
      CYFA_LAUNCH("token_bwd", s, (launch_k(token_bwd_kernel<256, __nv_bfloat16>, grid, 256, 0, s, p)));
    else
      CYFA_LAUNCH("token_bwd", s, (launch_k(token_bwd_kernel<128, __nv_bfloat16>, grid, 256, 0, s, p)));
  } else {
    if (K == 256) CYFA_LAUNCH("token_bwd", s, (launch_k(token_bwd_kernel<256, float>, grid, 256, 0, s, p)));
    else CYFA_LAUNCH("token_bwd", s, (launch_k(token_bwd_kernel<128, float>, grid, 256, 0, s, p)));
  }
  return launch_status();
}

}  // namespace cyfa

// Gate layout, clock scan and in-tile gate cumsum; `lengths` (or null) makes the
// tokens past each sequence's length neutral (right padding).
static int gates_fwd_launch(const float* g, const float* delta, const float* beta,
                            const float* clock0, float* G, float* lam, float* beta_h,
                            float* clock_out, int B, int T, int H, const int* lengths,
                            void* stream) {
  CYFA_REQUIRE(g && delta && beta && G && lam && beta_h, kNullPointer);
  CYFA_REQUIRE(B > 0 && T > 0 && H > 0, kBadShape);
  const int TP = (T + 127) / 128 * 128;
  GatesParams p{g, delta, beta, clock0, G, lam, beta_h, clock_out, B, T, H, TP, lengths};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CYFA_LAUNCH("gates_fwd", st,
              launch_k(gates_fwd_kernel, dim3(B * H, (TP + 1023) / 1024), 1024, 0, st, p));
  return launch_status();
}

extern "C" {

int cyfa_version(void) { return 1; }

const char* cyfa_strerror(int status) {
  switch (status) {
    case kOk: return "ok";
    case kBadShape: return "unsupported or inconsistent shape";
    case kNullPointer: return "required pointer is null";
    case kMisaligned: return "pointer or stride is not 16-byte aligned";
    case kBadDtype: return "unsupported dtype";
    case kNoDriver: return "CUDA driver entry point cuTensorMapEncodeTiled unavailable";
    case kTensorMap: return "cuTensorMapEncodeTiled rejected the tensor";
    case kWorkspace: return "workspace too small";
    default: break;
  }
  if (status < 0) return cudaGetErrorString(static_cast<cudaError_t>(-status));
  return "unknown status";
}

long long cyfa_launch_count(void) { return g_launches.load(); }

int cyfa_set_pdl(int on) { return g_pdl.exchange(on != 0 ? 1 : 0); }

int cyfa_set_scan_split(int on) { return g_scan_split.exchange(on != 0 ? 1 : 0); }

int cyfa_set_aux_stream(void* aux) {
  t_aux = static_cast<cudaStream_t>(aux);
  return 0;
}

int cyfa_profile_enable(int on) {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  for (auto& r : g_prof) {
    cudaEventDestroy(r.start);
    cudaEventDestroy(r.stop);
  }
  g_prof.clear();
  g_prof_on = on != 0;
  return 0;
}

int cyfa_profile_report(int max, const char** names, float* total_ms, int* counts) {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  int n = 0;
  for (auto& r : g_prof) {
    if (cudaEventSynchronize(r.stop) != cudaSuccess) return -1;
    float ms = 0.f;
    cudaEventElapsedTime(&ms, r.start, r.stop);
    int i = 0;
    while (i < n && names[i] != r.name) ++i;
    if (i == n) {
      if (n == max) continue;
      names[n] = r.name;
      total_ms[n] = 0.f;
      counts[n] = 0;
      ++n;
    }
    total_ms[i] += ms;
    counts[i] += 1;
  }
  return n;
}

int cyfa_device_error(int reset) {
  int v = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return -1;
  if (reset) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
  }
  return v;
}

int cyfa_selftest_umma(const void* a, const void* b, float* c, int K, int N, int a_mn, int b_mn,
                       void* stream) {
  CYFA_REQUIRE(a && b && c, kNullPointer);
  CYFA_REQUIRE(K >= 64 && K <= 256 && K % 64 == 0, kBadShape);
  CYFA_REQUIRE(N == 64 || N == 128 || N == 256, kBadShape);
  CUtensorMap ta, tb;
  int st = a_mn ? tmap_2d(&ta, a, K, 128, K) : tmap_2d(&ta, a, 128, K, 128);
  if (st) return st;
  st = b_mn ? tmap_2d(&tb, b, K, N, K) : tmap_2d(&tb, b, N, K, N);
  if (st) return st;
  SelftestParams p{K, N, a_mn ? 1 : 0, b_mn ? 1 : 0, c};
  const int smem = (128 + N) * K * 2 + 1024;
  cudaFuncSetAttribute(umma_selftest_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  cudaStream_t cs = static_cast<cudaStream_t>(stream);
  CYFA_LAUNCH("umma_selftest", cs, umma_selftest_kernel<<<1, 128, smem, cs>>>(ta, tb, p));
  return launch_status();
}

int cyfa_decode_step(const void* q, const void* k, const void* v, const float* g,
                     const float* delta, const float* beta, const float* table,
                     const float* q_norm_weight, const float* k_norm_weight, const float* hk_in,
                     const float* hv_in, const float* clock_in, float* hk_out, float* hv_out,
                     float* clock_out, void* out, int B, int H, int K, int V, int dtype,
                     float q_eps, float k_eps, float scale, void* stream) {
  CYFA_REQUIRE(q && k && v && g && delta && beta && table && q_norm_weight && k_norm_weight &&
                   hk_out && hv_out && clock_out && out,
               kNullPointer);
  CYFA_REQUIRE(B > 0 && H > 0 && (K == 128 || K == 256) && (V == 128 || V == 256), kBadShape);
  CYFA_REQUIRE(dtype == 0 || dtype == 1, kBadDtype);
  CYFA_REQUIRE(aligned(hk_out, 16) && aligned(hv_out, 16) && aligned(table, 16) &&
                   (!hk_in || aligned(hk_in, 16)) && (!hv_in || aligned(hv_in, 16)),
               kMisaligned);
  DecodeParams p{q, k, v, g, delta, beta, table, q_norm_weight, k_norm_weight, hk_in, hv_in,
                 clock_in, hk_out, hv_out, clock_out, out, B * H, H, q_eps, k_eps, scale};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid(B * H);
#define CYFA_DECODE(T, KK, VV) \
  CYFA_LAUNCH("decode_step", s, (launch_k(decode_step_kernel<T, KK, VV>, grid, 256, 0, s, p)))
  if (dtype == 0) {
    if (K == 256 && V == 256) CYFA_DECODE(__nv_bfloat16, 256, 256);
    else if (K == 128 && V == 128) CYFA_DECODE(__nv_bfloat16, 128, 128);
    else if (K == 256) CYFA_DECODE(__nv_bfloat16, 256, 128);
    else CYFA_DECODE(__nv_bfloat16, 128, 256);
  } else {
    if (K == 256 && V == 256) CYFA_DECODE(float, 256, 256);
    else if (K == 128 && V == 128) CYFA_DECODE(float, 128, 128);
    else if (K == 256) CYFA_DECODE(float, 256, 128);
    else CYFA_DECODE(float, 128, 256);
  }
#undef CYFA_DECODE
  return launch_status();
}

int cyfa_chunk_fwd_f32(const float* q, const float* k, const float* v, const float* g,
                       const float* delta, const float* beta, const float* table,
                       const float* q_norm_weight, const float* k_norm_weight, const float* hk0,
                       const float* hv0, const float* clock0, float* o, float* hk, float* hv,
                       float* clock, int B, int T, int H, int K, int V, float q_eps, float k_eps,
                       float scale, void* stream) {
  CYFA_REQUIRE(q && k && v && g && delta && beta && table && q_norm_weight && k_norm_weight &&
                   o && hk && hv && clock,
               kNullPointer);
  CYFA_REQUIRE(B > 0 && T >= 0 && H > 0 && (K == 128 || K == 256) && (V == 128 || V == 256),
               kBadShape);
  CYFA_REQUIRE(aligned(hk, 16) && aligned(hv, 16) && aligned(table, 16) &&
                   (!hk0 || aligned(hk0, 16)) && (!hv0 || aligned(hv0, 16)),
               kMisaligned);
  RecurrentParams p{q, k, v, g, delta, beta, table, q_norm_weight, k_norm_weight, hk0, hv0,
                    clock0, hk, hv, clock, o, B, T, H, q_eps, k_eps, scale};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid(B * H);
#define CYFA_REC(KK, VV) \
  CYFA_LAUNCH("recurrent_fwd_f32", s, (launch_k(recurrent_fwd_f32_kernel<KK, VV>, grid, 256, 0, s, p)))
  if (K == 256 && V == 256) CYFA_REC(256, 256);
  else if (K == 128 && V == 128) CYFA_REC(128, 128);
  else if (K == 256) CYFA_REC(256, 128);
  else CYFA_REC(128, 256);
#undef CYFA_REC
  return launch_status();
}

int cyfa_gates_fwd(const float* g, const float* delta, const float* beta, const float* clock0,
                   float* G, float* lam, float* beta_h, float* clock_out, int B, int T, int H,
                   void* stream) {
  return gates_fwd_launch(g, delta, beta, clock0, G, lam, beta_h, clock_out, B, T, H, nullptr,
                          stream);
}

int cyfa_token_fwd(const void* q, const void* k, const float* q_norm_weight,
                   const float* k_norm_weight, const float* lam, const float* beta_h, void* qn,
                   void* kn, void* w, float* q_rs, float* k_rs, int B, int T, int H, int K,
                   float q_eps, float k_eps, void* stream) {
  return token_fwd_launch(q, k, q_norm_weight, k_norm_weight, lam, beta_h, qn, kn, w, q_rs, k_rs,
                          B, T, H, K, q_eps, k_eps, (long long)H * K, (long long)H * K, stream);
}

int cyfa_token_bwd(const void* q, const void* k, const float* q_norm_weight,
                   const float* k_norm_weight, const float* q_rs, const float* k_rs,
                   const float* dqn, const float* dkn, const float* lam, const float* beta_h,
                   const float* dw, void* dq, void* dk, float* dqw_part, float* dkw_part,
                   float* dlam, float* dbeta_h, int B, int T, int H, int K, void* stream) {
  const long long d = (long long)H * K;
  return token_bwd_launch(q, k, q_norm_weight, k_norm_weight, q_rs, k_rs, dqn, dkn, lam, beta_h,
                          dw, nullptr, dq, dk, dqw_part, dkw_part, dlam, dbeta_h, B, T, H, K, d, d, d, d,
                          false, stream);
}

int cyfa_gates_bwd(const float* dG, const float* dlam, const float* dbeta_h, const float* dclock,
                   float* dg, float* ddelta, float* dbeta, float* dclock0, int B, int T, int H,
                   void* stream) {
  CYFA_REQUIRE(dG && dlam && dbeta_h && dg && ddelta && dbeta, kNullPointer);
  CYFA_REQUIRE(B > 0 && T > 0 && H > 0, kBadShape);
  const int TP = (T + 127) / 128 * 128;
  GatesBwdParams p{dG, 1, 0, dlam, nullptr, nullptr, nullptr, 0, 0, dbeta_h, dclock, dg, ddelta,
                   dbeta, dclock0, B, T, H, TP};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CYFA_LAUNCH("gates_bwd", st,
              launch_k(gates_bwd_kernel, dim3(B * H, (TP + 1023) / 1024), 1024, 0, st, p));
  return launch_status();
}

}  // extern "C"
