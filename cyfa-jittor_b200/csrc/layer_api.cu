// C-ABI of the layer glue kernels (short convolution, gate activations, gated
// output norm).  Work buffers for the deterministic weight-gradient partials are
// caller-owned; their sizes come from the *_work_bytes queries.
#include "../../include/cyfa.h"
#include "cyfa_common.cuh"

namespace cyfa {


static int gate_bwd_blocks(long long n) {
  const long long want = (n + 255) / 256;
  return int(want < 296 ? want : 296);
}

static int norm_bwd_blocks(int rows) {
  const int want = (rows + 7) / 8;
  return want < 296 ? want : 296;
}

}  // namespace cyfa

using namespace cyfa;

// [B, T, C] bf16 rows `stride` elements apart as a 3-D map {C, T, B} with a
// {128, kCtBoxRows, 1} unswizzled box (the short-convolution tiles).
static int conv_tmap(CUtensorMap* m, const void* base, int B, int T, int C, long long stride) {
  const uint64_t dims[3] = {uint64_t(C), uint64_t(T), uint64_t(B)};
  const uint64_t strides[2] = {uint64_t(stride) * 2, uint64_t(stride) * 2 * uint64_t(T)};
  const uint32_t box[3] = {128, uint32_t(kCtBoxRows), 1};
  return make_tmap_bf16(m, base, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
}

// Rows (token, head) x D bf16, dense, as the 3-D map {D, H, tokens} with a
// {D, 1, kNtRows} unswizzled box: one head's rows of kNtRows consecutive tokens.
static int norm_tmap(CUtensorMap* m, const void* base, int H, int BT, int D) {
  const uint64_t dims[3] = {uint64_t(D), uint64_t(H), uint64_t(BT)};
  const uint64_t strides[2] = {uint64_t(D) * 2, uint64_t(H) * D * 2};
  const uint32_t box[3] = {uint32_t(D), 1, uint32_t(kNtRows)};
  return make_tmap_bf16(m, base, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
}

template <int W>
static void conv_fwd_tma_launch(const CUtensorMap& mx, const ConvTmaParams& p, int grid,
                                cudaStream_t s) {
  set_smem(short_conv_fwd_tma_kernel<W>, kCtSmem);
  CYFA_LAUNCH("short_conv_fwd", s, launch_k(short_conv_fwd_tma_kernel<W>, grid, 288, kCtSmem, s, mx, p));
}

template <int W>
static void conv_bwd_tma_launch(const CUtensorMap& mx, const CUtensorMap& md,
                                const ConvTmaParams& p, int grid, cudaStream_t s) {
  set_smem(short_conv_bwd_tma_kernel<W>, kCtSmemB);
  CYFA_LAUNCH("short_conv_bwd", s,
              launch_k(short_conv_bwd_tma_kernel<W>, grid, 288, kCtSmemB, s, mx, md, p));
}

extern "C" {

size_t cyfa_short_conv_work_bytes(int B, int T, int C, int W) {
  if (B <= 0 || T <= 0 || C <= 0 || W < 1 || W > 4) return 0;
  return size_t(conv_bwd_rows(B, T)) * C * (W + 1) * sizeof(float);
}

int cyfa_short_conv_fwd(const void* x, long long x_stride, const void* cache, const float* w,
                        const float* bias, void* y, int B, int T, int C, int W, void* stream) {
  CYFA_REQUIRE(x && w && y, kNullPointer);
  CYFA_REQUIRE(B > 0 && T > 0 && C > 0 && C % 8 == 0 && W >= 1 && W <= 4 && x_stride >= C &&
                   x_stride % 8 == 0,
               kBadShape);
  CYFA_REQUIRE(aligned(x, 16) && aligned(y, 16) && (!cache || aligned(cache, 16)), kMisaligned);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CUtensorMap mx;
  if (!cache && C % 128 == 0 && conv_tmap(&mx, x, B, T, C, x_stride) == kOk) {
    // persistent CTAs (two per SM): channel block x token-tile group
    const int ncb = C / 128, nT = (T + kCtRows - 1) / kCtRows;
    int G = 296 / ncb;
    if (G < 1) G = 1;
    if (G > B * nT) G = B * nT;
    const int grid = ncb * G;
    ConvTmaParams q{B, T, C, nT, w, bias, static_cast<__nv_bfloat16*>(y), C, nullptr};
    switch (W) {
      case 1: conv_fwd_tma_launch<1>(mx, q, grid, s); break;
      case 2: conv_fwd_tma_launch<2>(mx, q, grid, s); break;
      case 3: conv_fwd_tma_launch<3>(mx, q, grid, s); break;
      default: conv_fwd_tma_launch<4>(mx, q, grid, s); break;
    }
    return launch_status();
  }
  ConvParams p{static_cast<const __nv_bfloat16*>(x), x_stride,
               static_cast<const __nv_bfloat16*>(cache), w, bias, static_cast<__nv_bfloat16*>(y),
               nullptr, nullptr, 0, nullptr, B, T, C};
  const dim3 grid((C + 127) / 128, (T + kConvWarps * kConvRun - 1) / (kConvWarps * kConvRun), B);
  switch (W) {
    case 1: CYFA_LAUNCH("short_conv_fwd", s, launch_k(short_conv_fwd_kernel<1>, grid, 256, 0, s, p)); break;
    case 2: CYFA_LAUNCH("short_conv_fwd", s, launch_k(short_conv_fwd_kernel<2>, grid, 256, 0, s, p)); break;
    case 3: CYFA_LAUNCH("short_conv_fwd", s, launch_k(short_conv_fwd_kernel<3>, grid, 256, 0, s, p)); break;
    default: CYFA_LAUNCH("short_conv_fwd", s, launch_k(short_conv_fwd_kernel<4>, grid, 256, 0, s, p)); break;
  }
  return launch_status();
}

int cyfa_short_conv_bwd(const void* x, long long x_stride, const float* w, const void* dy,
                        void* dx, long long dx_stride, float* dw, float* dbias, int B, int T,
                        int C, int W, void* work, size_t work_bytes, void* stream) {
  CYFA_REQUIRE(x && w && dy && dx && dw && work, kNullPointer);
  CYFA_REQUIRE(B > 0 && T > 0 && C > 0 && C % 8 == 0 && W >= 1 && W <= 4 && x_stride >= C &&
                   x_stride % 8 == 0 && dx_stride >= C && dx_stride % 8 == 0,
               kBadShape);
  CYFA_REQUIRE(work_bytes >= cyfa_short_conv_work_bytes(B, T, C, W), kWorkspace);
  CYFA_REQUIRE(aligned(x, 16) && aligned(dy, 16) && aligned(dx, 16), kMisaligned);
  float* part = static_cast<float*>(work);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rows = conv_bwd_rows(B, T);
  CUtensorMap mx, md;
  if (C % 128 == 0 && conv_tmap(&mx, x, B, T, C, x_stride) == kOk &&
      conv_tmap(&md, dy, B, T, C, C) == kOk) {
    // persistent CTAs (two per SM): channel block x token-tile group; one partial
    // row per group
    const int ncb = C / 128, nT = (T + kCtRows - 1) / kCtRows;
    int G = 296 / ncb;
    if (G < 1) G = 1;
    if (G > rows) G = rows;
    if (G > B * nT) G = B * nT;
    rows = G;
    ConvTmaParams q{B, T, C, nT, w, nullptr, static_cast<__nv_bfloat16*>(dx), dx_stride, part};
    switch (W) {
      case 1: conv_bwd_tma_launch<1>(mx, md, q, ncb * G, s); break;
      case 2: conv_bwd_tma_launch<2>(mx, md, q, ncb * G, s); break;
      case 3: conv_bwd_tma_launch<3>(mx, md, q, ncb * G, s); break;
      default: conv_bwd_tma_launch<4>(mx, md, q, ncb * G, s); break;
    }
  } else {
    ConvParams p{static_cast<const __nv_bfloat16*>(x), x_stride, nullptr, w, nullptr, nullptr,
                 static_cast<const __nv_bfloat16*>(dy), static_cast<__nv_bfloat16*>(dx), dx_stride,
                 part, B, T, C};
    const dim3 grid((C + 127) / 128, rows);
    switch (W) {
    case 1: CYFA_LAUNCH("short_conv_bwd", s, (launch_k(short_conv_bwd_kernel<1>, grid, 256, 0, s, p))); break;
    case 2: CYFA_LAUNCH("short_conv_bwd", s, (launch_k(short_conv_bwd_kernel<2>, grid, 256, 0, s, p))); break;
    case 3: CYFA_LAUNCH("short_conv_bwd", s, (launch_k(short_conv_bwd_kernel<3>, grid, 256, 0, s, p))); break;
    default: CYFA_LAUNCH("short_conv_bwd", s, (launch_k(short_conv_bwd_kernel<4>, grid, 256, 0, s, p))); break;
    }
  }
  int rc = launch_status();
  if (rc) return rc;
  // reduce the partial rows: columns are [c][0..W-1] = dw, [c][W] = dbias
  const int cols = C * (W + 1);
  cudaStream_t sr = defer_stream(s);
  CYFA_LAUNCH("conv_param_sum", sr,
              (launch_k(conv_param_sum_kernel, (cols + 255) / 256, 256, 0, sr, part, rows, C, W, dw,
                        dbias)));
  return launch_status();
}

int cyfa_gate_act_fwd(const void* a, long long a_stride, const void* b, long long b_stride,
                      const void* d, long long d_stride, const float* A_log,
                      const float* dt_bias, const float* b_bias, const float* d_bias, float* g,
                      float* delta, float* beta, int rows, int H, void* stream) {
  CYFA_REQUIRE(a && b && d && A_log && dt_bias && g && delta && beta, kNullPointer);
  CYFA_REQUIRE(rows > 0 && H > 0 && 256 % H == 0 && a_stride >= H && b_stride >= H &&
                   d_stride >= H,
               kBadShape);
  GateActParams p{static_cast<const __nv_bfloat16*>(a), a_stride,
                  static_cast<const __nv_bfloat16*>(b), b_stride,
                  static_cast<const __nv_bfloat16*>(d), d_stride, A_log, dt_bias, b_bias, d_bias, g,
                  delta, beta, nullptr, nullptr, nullptr, nullptr, 0, nullptr, 0, nullptr, 0,
                  nullptr, rows, H};
  const long long n = (long long)rows * H;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CYFA_LAUNCH("gate_act_fwd", s,
              (launch_k(gate_act_fwd_kernel, unsigned((n + 255) / 256), 256, 0, s, p)));
  return launch_status();
}

size_t cyfa_gate_act_work_bytes(int rows, int H) {
  if (rows <= 0 || H <= 0) return 0;
  return size_t(gate_bwd_blocks((long long)rows * H)) * 4 * H * sizeof(float);
}

int cyfa_gate_act_bwd(const void* a, long long a_stride, const void* b, long long b_stride,
                      const void* d, long long d_stride, const float* A_log,
                      const float* dt_bias, const float* b_bias, const float* d_bias,
                      const float* dg, const float* ddelta, const float* dbeta, void* da,
                      long long da_stride, void* db, long long db_stride, void* dd,
                      long long dd_stride, float* dA_log, float* ddt_bias, float* db_bias,
                      float* dd_bias, int rows, int H, void* work, size_t work_bytes,
                      void* stream) {
  CYFA_REQUIRE(a && b && d && A_log && dt_bias && dg && ddelta && dbeta && da && db && dd &&
                   dA_log && ddt_bias && work,
               kNullPointer);
  CYFA_REQUIRE(rows > 0 && H > 0 && 256 % H == 0, kBadShape);
  CYFA_REQUIRE(work_bytes >= cyfa_gate_act_work_bytes(rows, H), kWorkspace);
  float* part = static_cast<float*>(work);
  GateActParams p{static_cast<const __nv_bfloat16*>(a), a_stride,
                  static_cast<const __nv_bfloat16*>(b), b_stride,
                  static_cast<const __nv_bfloat16*>(d), d_stride, A_log, dt_bias, b_bias, d_bias,
                  nullptr, nullptr, nullptr, dg, ddelta, dbeta, static_cast<__nv_bfloat16*>(da),
                  da_stride,
                  static_cast<__nv_bfloat16*>(db), db_stride, static_cast<__nv_bfloat16*>(dd),
                  dd_stride, part, rows, H};
  const int nblk = gate_bwd_blocks((long long)rows * H);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CYFA_LAUNCH("gate_act_bwd", s, (launch_k(gate_act_bwd_kernel, nblk, 256, 0, s, p)));
  int rc = launch_status();
  if (rc) return rc;
  // partial columns: dA_log | ddt_bias | db_bias | dd_bias, each H wide
  cudaStream_t sr = defer_stream(s);
  CYFA_LAUNCH("column_sum", sr,
              (launch_k(gate_param_sum_kernel, 1, 1024, 0, sr, part, nblk, H, dA_log, ddt_bias,
                        db_bias, dd_bias)));
  return launch_status();
}

int cyfa_gated_norm_fwd(const void* x, const void* gate, const float* w, float eps, float scale,
                        void* y, float* rstd, int rows, int D, void* stream) {
  CYFA_REQUIRE(aligned(w, 16), kMisaligned);
  CYFA_REQUIRE(x && gate && w && y && rstd, kNullPointer);
  CYFA_REQUIRE(rows > 0 && (D == 256 || D == 128), kBadShape);
  CYFA_REQUIRE(aligned(x, 16) && aligned(gate, 16) && aligned(y, 16), kMisaligned);
  GatedNormParams p{static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(gate),
                    w, eps, scale, static_cast<__nv_bfloat16*>(y), rstd, nullptr, nullptr, nullptr,
                    nullptr, rows};
  const unsigned grid = unsigned(norm_fwd_blocks(rows, 1));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (D == 256) CYFA_LAUNCH("gated_norm_fwd", s, (launch_k(gated_norm_fwd_kernel<8>, grid, 256, 0, s, p)));
  else CYFA_LAUNCH("gated_norm_fwd", s, (launch_k(gated_norm_fwd_kernel<4>, grid, 256, 0, s, p)));
  return launch_status();
}

size_t cyfa_gated_norm_work_bytes(int rows, int D) {
  if (rows <= 0 || D <= 0) return 0;
  return size_t(norm_bwd_blocks(rows)) * D * sizeof(float);
}

int cyfa_gated_norm_bwd(const void* x, const void* gate, const float* w, float scale,
                        const float* rstd, const void* dy, void* dx, void* dgate, float* dw,
                        int rows, int D, void* work, size_t work_bytes, void* stream) {
  CYFA_REQUIRE(aligned(w, 16), kMisaligned);
  CYFA_REQUIRE(x && gate && w && rstd && dy && dx && dgate && dw && work, kNullPointer);
  CYFA_REQUIRE(rows > 0 && (D == 256 || D == 128), kBadShape);
  CYFA_REQUIRE(work_bytes >= cyfa_gated_norm_work_bytes(rows, D), kWorkspace);
  float* part = static_cast<float*>(work);
  GatedNormParams p{static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(gate),
                    w, 0.f, scale, nullptr, const_cast<float*>(rstd),
                    static_cast<const __nv_bfloat16*>(dy), static_cast<__nv_bfloat16*>(dx),
                    static_cast<__nv_bfloat16*>(dgate), part, rows};
  const int nblk = norm_bwd_blocks(rows);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (D == 256) CYFA_LAUNCH("gated_norm_bwd", s, (launch_k(gated_norm_bwd_kernel<8>, nblk, 256, 0, s, p)));
  else CYFA_LAUNCH("gated_norm_bwd", s, (launch_k(gated_norm_bwd_kernel<4>, nblk, 256, 0, s, p)));
  int rc = launch_status();
  if (rc) return rc;
  cudaStream_t sr = defer_stream(s);
  CYFA_LAUNCH("column_sum", sr,
              (launch_k(column_sum_kernel, (D + 31) / 32, 1024, 0, sr, part, dw, nblk, D, nullptr,
                        nullptr, 0x7fffffff, nullptr)));
  return launch_status();
}

int cyfa_gated_norm_bias_fwd(const void* x, const void* gate, const void* gate_bias, int H,
                             const float* w, float eps, float scale, void* y, float* rstd,
                             int rows, int D, void* stream) {
  CYFA_REQUIRE(aligned(w, 16), kMisaligned);
  CYFA_REQUIRE(x && gate && gate_bias && w && y && rstd, kNullPointer);
  CYFA_REQUIRE(rows > 0 && H > 0 && rows % H == 0 && (D == 256 || D == 128), kBadShape);
  CYFA_REQUIRE(aligned(x, 16) && aligned(gate, 16) && aligned(y, 16) && aligned(gate_bias, 16),
               kMisaligned);
  GatedNormParams p{static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(gate),
                    w, eps, scale, static_cast<__nv_bfloat16*>(y), rstd, nullptr, nullptr, nullptr,
                    nullptr, rows, static_cast<const __nv_bfloat16*>(gate_bias), H, 0};
  unsigned grid = unsigned(norm_fwd_blocks(rows, H));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CUtensorMap mx, mg;
  const int BT = rows / H;
  if (norm_tmap(&mx, x, H, BT, D) == kOk && norm_tmap(&mg, gate, H, BT, D) == kOk) {
    int G = 296 / H;  // persistent CTAs (two per SM): head x token-tile group
    if (G > (BT + kNtRows - 1) / kNtRows) G = (BT + kNtRows - 1) / kNtRows;
    if (G < 1) G = 1;
    grid = unsigned(H * G);
    if (D == 256) {
      set_smem(gated_norm_fwd_tma_kernel<8>, norm_fwd_tma_smem<8>());
      CYFA_LAUNCH("gated_norm_fwd", s, (launch_k(gated_norm_fwd_tma_kernel<8>, grid, 288,
                                                 norm_fwd_tma_smem<8>(), s, mx, mg, p)));
    } else {
      set_smem(gated_norm_fwd_tma_kernel<4>, norm_fwd_tma_smem<4>());
      CYFA_LAUNCH("gated_norm_fwd", s, (launch_k(gated_norm_fwd_tma_kernel<4>, grid, 288,
                                                 norm_fwd_tma_smem<4>(), s, mx, mg, p)));
    }
  } else if (D == 256) {
    CYFA_LAUNCH("gated_norm_fwd", s, (launch_k(gated_norm_fwd_kernel<8>, grid, 256, 0, s, p)));
  } else {
    CYFA_LAUNCH("gated_norm_fwd", s, (launch_k(gated_norm_fwd_kernel<4>, grid, 256, 0, s, p)));
  }
  return launch_status();
}

// Block count of the biased backward: three per SM, a multiple of H (each warp
// stays on one head).
static int norm_bias_bwd_blocks(int rows, int H) {
  int n = (rows + 7) / 8;
  if (n > 444) n = 444;
  n -= n % H;
  return n < H ? H : n;
}

size_t cyfa_gated_norm_bias_work_bytes(int rows, int D, int H) {
  if (rows <= 0 || D <= 0 || H <= 0) return 0;
  return size_t(norm_bias_bwd_blocks(rows, H)) * size_t(D + H * D) * sizeof(float);
}

int cyfa_gated_norm_bias_bwd(const void* x, const void* gate, const void* gate_bias, int H,
                             const float* w, float scale, const float* rstd, const void* dy,
                             void* dx, void* dgate, float* dw, float* dgate_bias, int rows, int D,
                             void* work, size_t work_bytes, void* stream) {
  CYFA_REQUIRE(aligned(w, 16), kMisaligned);
  CYFA_REQUIRE(x && gate && gate_bias && w && rstd && dy && dx && dgate && dw && dgate_bias && work,
               kNullPointer);
  CYFA_REQUIRE(rows > 0 && H > 0 && rows % H == 0 && (D == 256 || D == 128), kBadShape);
  CYFA_REQUIRE(aligned(gate_bias, 16), kMisaligned);
  CYFA_REQUIRE(work_bytes >= cyfa_gated_norm_bias_work_bytes(rows, D, H), kWorkspace);
  float* part = static_cast<float*>(work);
  const int cols = D + H * D;
  GatedNormParams p{static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(gate),
                    w, 0.f, scale, nullptr, const_cast<float*>(rstd),
                    static_cast<const __nv_bfloat16*>(dy), static_cast<__nv_bfloat16*>(dx),
                    static_cast<__nv_bfloat16*>(dgate), part, rows,
                    static_cast<const __nv_bfloat16*>(gate_bias), H, cols};
  int nblk = norm_bias_bwd_blocks(rows, H);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CUtensorMap mx, mg, md;
  const int BT = rows / H;
  if (norm_tmap(&mx, x, H, BT, D) == kOk && norm_tmap(&mg, gate, H, BT, D) == kOk &&
      norm_tmap(&md, dy, H, BT, D) == kOk) {
    // persistent CTAs: head x token-tile group (G groups per head)
    int G = 148 / H;
    if (G > (BT + kNtRows - 1) / kNtRows) G = (BT + kNtRows - 1) / kNtRows;
    if (G > nblk / H) G = nblk / H;
    if (G < 1) G = 1;
    nblk = H * G;
    if (D == 256) {
      set_smem(gated_norm_bwd_tma_kernel<8>, norm_bwd_tma_smem<8>());
      CYFA_LAUNCH("gated_norm_bwd", s, (launch_k(gated_norm_bwd_tma_kernel<8>, nblk, 288,
                                                 norm_bwd_tma_smem<8>(), s, mx, mg, md, p)));
    } else {
      set_smem(gated_norm_bwd_tma_kernel<4>, norm_bwd_tma_smem<4>());
      CYFA_LAUNCH("gated_norm_bwd", s, (launch_k(gated_norm_bwd_tma_kernel<4>, nblk, 288,
                                                 norm_bwd_tma_smem<4>(), s, mx, mg, md, p)));
    }
  } else if (D == 256) {
    CYFA_LAUNCH("gated_norm_bwd", s, (launch_k(gated_norm_bwd_kernel<8>, nblk, 256, 0, s, p)));
  } else {
    CYFA_LAUNCH("gated_norm_bwd", s, (launch_k(gated_norm_bwd_kernel<4>, nblk, 256, 0, s, p)));
  }
  int rc = launch_status();
  if (rc) return rc;
  cudaStream_t sr = defer_stream(s);
  CYFA_LAUNCH("column_sum", sr,
              (launch_k(column_sum_kernel, (cols + 31) / 32, 1024, 0, sr, part, dw, nblk, cols,
                        nullptr, nullptr, D, dgate_bias)));
  return launch_status();
}

}  // extern "C"
