// Layer glue kernels around the CyFA op, replacing the reference layer's
// elementwise paths (cyclic_flow_attention/layers/cyfa.py):
//   short_conv_fwd/bwd : causal depthwise convolution without activation
//                        (ShortConvolution :138-233), bf16 in/out, fp32 accumulate
//   gate_act_fwd/bwd   : g = -exp(A_log) softplus(a + dt_bias), delta = sigmoid(d),
//                        beta = sigmoid(b) (:323-326)
//   gated_norm_fwd/bwd : RMSNorm(scale * o) * w * sigmoid(gate) over head_v_dim
//                        (o_norm(o * (num_slots - 1), gate), :350 and RMSNorm :62-135)
// All weight/bias gradients are written as per-block partial rows and reduced in
// a fixed order (column_sum_kernel), so the backward pass is deterministic.
#include "cyfa_common.cuh"

namespace cyfa {

// ============================================================ short conv
struct ConvParams {
  const __nv_bfloat16* x;     // [B, T, C] with token stride x_stride
  long long x_stride;
  const __nv_bfloat16* cache; // [B, W-1, C] history before t = 0, or null (zeros)
  const float* w;             // [C, W]
  const float* bias;          // [C] or null
  __nv_bfloat16* y;           // [B, T, C] dense
  const __nv_bfloat16* dy;    // backward: [B, T, C] dense
  __nv_bfloat16* dx;          // backward: [B, T, C] with token stride dx_stride
  long long dx_stride;
  float* part;                // backward: [gridDim.y * B, C * (W + 1)] partial dw | dbias
  int B, T, C;
};

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float* f) {
  unpack_bf16x8(*reinterpret_cast<const uint4*>(p), f);
}
__device__ __forceinline__ void store8(__nv_bfloat16* p, const float* f) {
  *reinterpret_cast<uint4*>(p) = make_uint4(pack_bf16(f[0], f[1]), pack_bf16(f[2], f[3]),
                                            pack_bf16(f[4], f[5]), pack_bf16(f[6], f[7]));
}

// Tiled short convolution.  A CTA of 256 threads owns 256 channels; a chunk of
// tokens (plus the W-1 halo rows) is staged in shared memory with asynchronous
// 16-byte copies, and thread (cg, run) computes channels 8cg..8cg+7 of the run's
// tokens.  Weights are staged once per CTA.  The backward CTA walks a token range
// with double-buffered staging.
constexpr int kConvChunk = 64;       // forward tokens per CTA
constexpr int kConvBwdChunk = 32;    // backward tokens per staged chunk
constexpr int kConvSplit = 8;        // backward token ranges per (channel block, batch)

// Issues async copies of rows row0 .. row0 + nrows - 1 (token index) of src,
// channels c_base .. +255, into tile (row-major [nrows][256] bf16).
template <int W>
__device__ __forceinline__ void conv_stage_rows(uint8_t* tile, const __nv_bfloat16* src,
                                                long long stride, int b, int T, int C,
                                                int c_base, int row0, int nrows,
                                                const __nv_bfloat16* cache) {
  const uint32_t base = smem_u32(tile);
  for (int idx = threadIdx.x; idx < nrows * 32; idx += blockDim.x) {
    const int r = idx >> 5, cg = idx & 31;
    const int t = row0 + r, c = c_base + cg * 8;
    const __nv_bfloat16* g = src;
    bool valid = false;
    if (c < C) {
      if (t >= 0 && t < T) {
        g = src + (size_t(b) * T + t) * stride + c;
        valid = true;
      } else if (t < 0 && cache) {
        g = cache + (size_t(b) * (W - 1) + (W - 1) + t) * C + c;
        valid = true;
      }
    }
    cp_async16(base + r * 512 + cg * 16, g, valid);
  }
}

template <int W>
__global__ void __launch_bounds__(256) short_conv_fwd_kernel(ConvParams p) {
  __shared__ __align__(16) __nv_bfloat16 xs[kConvChunk + W - 1][256];
  __shared__ float ws[256][W + 1];
  const int c_base = blockIdx.x * 256, b = blockIdx.z;
  const int t0 = blockIdx.y * kConvChunk;
  conv_stage_rows<W>(reinterpret_cast<uint8_t*>(xs), p.x, p.x_stride, b, p.T, p.C, c_base,
                     t0 - (W - 1), kConvChunk + W - 1, p.cache);
  cp_async_commit();
  for (int i = threadIdx.x; i < 256 * W; i += 256) {
    const int c = c_base + i / W;
    ws[i / W][i % W] = c < p.C ? p.w[size_t(c) * W + i % W] : 0.f;
  }
  {
    const int c = c_base + threadIdx.x;
    ws[threadIdx.x][W] = (p.bias && c < p.C) ? p.bias[c] : 0.f;
  }
  cp_async_wait<0>();
  __syncthreads();
  const int cg = threadIdx.x & 31, run = threadIdx.x >> 5;
  const int c0 = c_base + cg * 8;
  if (c0 >= p.C) return;
  float wr[W][8], bias[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
#pragma unroll
    for (int i = 0; i < W; ++i) wr[i][e] = ws[cg * 8 + e][i];
    bias[e] = ws[cg * 8 + e][W];
  }
#pragma unroll
  for (int tt = 0; tt < 8; ++tt) {
    const int r = run * 8 + tt;  // output token t0 + r uses staged rows r .. r + W - 1
    const int t = t0 + r;
    float y[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) y[e] = bias[e];
#pragma unroll
    for (int i = 0; i < W; ++i) {
      float x[8];
      unpack_bf16x8(*reinterpret_cast<const uint4*>(&xs[r + i][cg * 8]), x);
#pragma unroll
      for (int e = 0; e < 8; ++e) y[e] += wr[i][e] * x[e];
    }
    if (t < p.T) store8(p.y + (size_t(b) * p.T + t) * p.C + c0, y);
  }
}

template <int W>
constexpr int conv_bwd_stage_bytes() {
  return 2 * (kConvBwdChunk + W - 1) * 512;  // x rows + dy rows
}
template <int W>
constexpr int conv_bwd_smem() {
  return 2 * conv_bwd_stage_bytes<W>() > 8 * 256 * (W + 1) * 4 ? 2 * conv_bwd_stage_bytes<W>()
                                                               : 8 * 256 * (W + 1) * 4;
}

// dx[tau] = sum_i w_i dy[tau + (W-1) - i];  dw_i = sum_t dy[t] x[t + i - (W-1)];  db = sum_t dy[t]
// grid (C/256, B * kConvSplit): each CTA walks one token range in chunks.
template <int W>
__global__ void __launch_bounds__(256) short_conv_bwd_kernel(ConvParams p) {
  extern __shared__ __align__(16) uint8_t conv_smem[];
  __shared__ float ws[256][W];
  constexpr int R = kConvBwdChunk + W - 1;  // staged rows per tile
  const int c_base = blockIdx.x * 256;
  const int b = blockIdx.y / kConvSplit, split = blockIdx.y % kConvSplit;
  const int nchunks = (p.T + kConvBwdChunk - 1) / kConvBwdChunk;
  const int per = (nchunks + kConvSplit - 1) / kConvSplit;
  const int k0 = split * per, k1 = min(nchunks, k0 + per);
  auto stage = [&](int kc, int buf) {
    uint8_t* base = conv_smem + buf * conv_bwd_stage_bytes<W>();
    const int t0 = kc * kConvBwdChunk;
    conv_stage_rows<W>(base, p.x, p.x_stride, b, p.T, p.C, c_base, t0 - (W - 1), R, nullptr);
    conv_stage_rows<W>(base + R * 512, p.dy, p.C, b, p.T, p.C, c_base, t0, R, nullptr);
    cp_async_commit();
  };
  if (k0 < k1) stage(k0, 0);
  for (int i = threadIdx.x; i < 256 * W; i += 256) {
    const int c = c_base + i / W;
    ws[i / W][i % W] = c < p.C ? p.w[size_t(c) * W + i % W] : 0.f;
  }
  __syncthreads();
  const int cg = threadIdx.x & 31, run = threadIdx.x >> 5;
  const int c0 = c_base + cg * 8;
  float wr[W][8];
#pragma unroll
  for (int e = 0; e < 8; ++e)
#pragma unroll
    for (int i = 0; i < W; ++i) wr[i][e] = ws[cg * 8 + e][i];
  float acc[W + 1][8];
#pragma unroll
  for (int i = 0; i <= W; ++i)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[i][e] = 0.f;
  for (int kc = k0; kc < k1; ++kc) {
    const int buf = (kc - k0) & 1;
    if (kc + 1 < k1) {
      stage(kc + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint8_t* base = conv_smem + buf * conv_bwd_stage_bytes<W>();
    auto xrow = [&](int r) { return reinterpret_cast<const uint4*>(base + r * 512 + cg * 16); };
    auto drow = [&](int r) {
      return reinterpret_cast<const uint4*>(base + R * 512 + r * 512 + cg * 16);
    };
    const int t0 = kc * kConvBwdChunk;
    if (c0 < p.C) {
#pragma unroll
      for (int tt = 0; tt < kConvBwdChunk / 8; ++tt) {
        const int r = run * (kConvBwdChunk / 8) + tt;
        const int t = t0 + r;
        float dy0[8], dx[8];
        unpack_bf16x8(*drow(r), dy0);
#pragma unroll
        for (int e = 0; e < 8; ++e) dx[e] = 0.f;
#pragma unroll
        for (int i = 0; i < W; ++i) {
          float d[8], x[8];
          unpack_bf16x8(*drow(r + W - 1 - i), d);
          unpack_bf16x8(*xrow(r + i), x);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            dx[e] += wr[i][e] * d[e];
            acc[i][e] += dy0[e] * x[e];
          }
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[W][e] += dy0[e];
        if (t < p.T) store8(p.dx + (size_t(b) * p.T + t) * p.dx_stride + c0, dx);
      }
    }
    __syncthreads();
  }
  // reduce the 8 runs through shared memory in a fixed order
  float* red = reinterpret_cast<float*>(conv_smem);  // 8 * 256 * (W+1) floats
#pragma unroll
  for (int i = 0; i <= W; ++i)
#pragma unroll
    for (int e = 0; e < 8; ++e) red[(run * 256 + cg * 8 + e) * (W + 1) + i] = acc[i][e];
  __syncthreads();
  const size_t prow = blockIdx.y;
  for (int idx = threadIdx.x; idx < 256 * (W + 1); idx += 256) {
    const int c = c_base + idx / (W + 1);
    if (c >= p.C) continue;
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) sum += red[k * 256 * (W + 1) + idx];
    p.part[prow * (size_t(p.C) * (W + 1)) + size_t(c) * (W + 1) + idx % (W + 1)] = sum;
  }
}

// ============================================================ gate activations
struct GateActParams {
  const __nv_bfloat16* a;  // a_proj output, token stride a_stride, H columns
  long long a_stride;
  const __nv_bfloat16* b;  // b_proj output (bias included)
  long long b_stride;
  const __nv_bfloat16* d;  // d_proj output (bias included)
  long long d_stride;
  const float* A_log;      // [H]
  const float* dt_bias;    // [H]
  const float* b_bias;     // [H] added to b, or null
  const float* d_bias;     // [H] added to d, or null
  float* g;                // [rows, H]
  float* delta;
  float* beta;
  // backward
  const float* dg;
  const float* ddelta;
  const float* dbeta;
  __nv_bfloat16* da;       // token stride da_stride
  long long da_stride;
  __nv_bfloat16* db;
  long long db_stride;
  __nv_bfloat16* dd;
  long long dd_stride;
  float* part;             // [gridDim.x, 4H]: dA_log | ddt_bias | db_bias | dd_bias
  int rows, H;
};

__device__ __forceinline__ float softplus_f(float x) {
  return x > 20.f ? x : log1pf(expf(x));  // torch softplus, beta 1, threshold 20
}
__device__ __forceinline__ float sigmoid_f(float x) { return 1.f / (1.f + expf(-x)); }

__global__ void __launch_bounds__(256) gate_act_fwd_kernel(GateActParams p) {
  const size_t i = size_t(blockIdx.x) * 256 + threadIdx.x;
  if (i >= size_t(p.rows) * p.H) return;
  const size_t r = i / p.H;
  const int h = int(i % p.H);
  const float a = __bfloat162float(p.a[r * p.a_stride + h]) + p.dt_bias[h];
  p.g[i] = -expf(p.A_log[h]) * softplus_f(a);
  p.delta[i] = sigmoid_f(__bfloat162float(p.d[r * p.d_stride + h]) + (p.d_bias ? p.d_bias[h] : 0.f));
  p.beta[i] = sigmoid_f(__bfloat162float(p.b[r * p.b_stride + h]) + (p.b_bias ? p.b_bias[h] : 0.f));
}

// One thread per (row, head); grid-strided; per-block fixed-order partial sums.
__global__ void __launch_bounds__(256) gate_act_bwd_kernel(GateActParams p) {
  __shared__ float red[256][4];
  const int h = threadIdx.x % p.H;  // H divides 256 (checked on the host)
  float sA = 0.f, sdt = 0.f, sb = 0.f, sd = 0.f;
  const size_t n = size_t(p.rows) * p.H;
  for (size_t i = size_t(blockIdx.x) * 256 + threadIdx.x; i < n; i += size_t(gridDim.x) * 256) {
    const size_t r = i / p.H;
    const float a = __bfloat162float(p.a[r * p.a_stride + h]) + p.dt_bias[h];
    const float eA = expf(p.A_log[h]);
    const float gv = -eA * softplus_f(a);
    const float dgv = p.dg[i];
    const float da = dgv * (-eA) * sigmoid_f(a);
    sA += dgv * gv;
    sdt += da;
    p.da[r * p.da_stride + h] = __float2bfloat16_rn(da);
    const float de = sigmoid_f(__bfloat162float(p.d[r * p.d_stride + h]) +
                               (p.d_bias ? p.d_bias[h] : 0.f));
    const float ddv = p.ddelta[i] * de * (1.f - de);
    p.dd[r * p.dd_stride + h] = __float2bfloat16_rn(ddv);
    const float be = sigmoid_f(__bfloat162float(p.b[r * p.b_stride + h]) +
                               (p.b_bias ? p.b_bias[h] : 0.f));
    const float dbv = p.dbeta[i] * be * (1.f - be);
    p.db[r * p.db_stride + h] = __float2bfloat16_rn(dbv);
    sb += dbv;
    sd += ddv;
  }
  red[threadIdx.x][0] = sA;
  red[threadIdx.x][1] = sdt;
  red[threadIdx.x][2] = sb;
  red[threadIdx.x][3] = sd;
  __syncthreads();
  if (threadIdx.x < p.H) {
    float x[4] = {0.f, 0.f, 0.f, 0.f};
    for (int t = threadIdx.x; t < 256; t += p.H)
#pragma unroll
      for (int k = 0; k < 4; ++k) x[k] += red[t][k];
#pragma unroll
    for (int k = 0; k < 4; ++k) p.part[size_t(blockIdx.x) * 4 * p.H + k * p.H + threadIdx.x] = x[k];
  }
}

// ============================================================ gated RMSNorm
struct GatedNormParams {
  const __nv_bfloat16* x;     // [rows, D]
  const __nv_bfloat16* gate;  // [rows, D]
  const float* w;             // [D]
  float eps, scale;
  __nv_bfloat16* y;           // [rows, D]
  float* rstd;                // [rows]
  const __nv_bfloat16* dy;    // backward
  __nv_bfloat16* dx;
  __nv_bfloat16* dgate;
  float* part;                // [gridDim.x, part_cols] partials: weight [D] | gate bias [H*D]
  int rows;
  const __nv_bfloat16* gbias = nullptr;  // optional gate bias [H*D]; rows are (token, head)
  int H = 1;                             // heads per token (rows % H = head)
  int part_cols = 0;                     // 0: D (no bias partials); else D + H*D
};

// One warp per row (grid-strided), D = 32 * E.
template <int E>
__global__ void __launch_bounds__(256) gated_norm_fwd_kernel(GatedNormParams p) {
  constexpr int D = 32 * E;
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= p.rows) return;
  float x[E], g[E];
  if constexpr (E == 8) {
    load8(p.x + size_t(row) * D + lane * 8, x);
    load8(p.gate + size_t(row) * D + lane * 8, g);
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e) {
      x[e] = __bfloat162float(p.x[size_t(row) * D + lane * E + e]);
      g[e] = __bfloat162float(p.gate[size_t(row) * D + lane * E + e]);
    }
  }
  if (p.gbias) {
    float b[E];
    load_bf16_vec<E>(p.gbias + size_t(row % p.H) * D + lane * E, b);
#pragma unroll
    for (int e = 0; e < E; ++e) g[e] += b[e];
  }
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    x[e] *= p.scale;
    ss += x[e] * x[e];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float rs = rsqrtf(ss / D + p.eps);
  if (lane == 0) p.rstd[row] = rs;
  float y[E];
#pragma unroll
  for (int e = 0; e < E; ++e) y[e] = x[e] * rs * p.w[lane * E + e] * sigmoid_f(g[e]);
  if constexpr (E == 8) {
    store8(p.y + size_t(row) * D + lane * 8, y);
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e) p.y[size_t(row) * D + lane * E + e] = __float2bfloat16_rn(y[e]);
  }
}

// With a gate bias the grid is a multiple of H, so every warp's rows belong to
// one head ((blockIdx.x * 8 + warp) % H) and its bias-gradient partial stays in
// registers; the block's per-head sums are formed in a fixed warp order.
template <int E>
__global__ void __launch_bounds__(256) gated_norm_bwd_kernel(GatedNormParams p) {
  constexpr int D = 32 * E;
  __shared__ float red[8][D];
  __shared__ float red_b[8][D];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const bool has_b = p.gbias != nullptr;
  float acc[E], acc_b[E], bias[E];
#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] = acc_b[e] = bias[e] = 0.f;
  if (has_b) load_bf16_vec<E>(p.gbias + size_t((blockIdx.x * 8 + wid) % p.H) * D + lane * E, bias);
  for (int row = blockIdx.x * 8 + wid; row < p.rows; row += gridDim.x * 8) {
    float x[E], g[E], dy[E];
    load_bf16_vec<E>(p.x + size_t(row) * D + lane * E, x);
    load_bf16_vec<E>(p.gate + size_t(row) * D + lane * E, g);
    load_bf16_vec<E>(p.dy + size_t(row) * D + lane * E, dy);
#pragma unroll
    for (int e = 0; e < E; ++e) g[e] += bias[e];
#pragma unroll
    for (int e = 0; e < E; ++e) x[e] *= p.scale;
    const float rs = p.rstd[row];
    float dn[E], n[E], dgv[E], dot = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float sg = sigmoid_f(g[e]), wv = p.w[lane * E + e];
      n[e] = x[e] * rs;
      const float z = n[e] * wv;
      dgv[e] = dy[e] * z * sg * (1.f - sg);
      const float dz = dy[e] * sg;
      acc[e] += dz * n[e];
      dn[e] = dz * wv;
      dot += dn[e] * n[e];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    dot /= D;
    float dxv[E];
#pragma unroll
    for (int e = 0; e < E; ++e) dxv[e] = p.scale * rs * (dn[e] - n[e] * dot);
    store_bf16_vec<E>(p.dx + size_t(row) * D + lane * E, dxv);
    store_bf16_vec<E>(p.dgate + size_t(row) * D + lane * E, dgv);
#pragma unroll
    for (int e = 0; e < E; ++e) acc_b[e] += dgv[e];
  }
#pragma unroll
  for (int e = 0; e < E; ++e) {
    red[wid][lane * E + e] = acc[e];
    red_b[wid][lane * E + e] = acc_b[e];
  }
  __syncthreads();
  const int pc = p.part_cols > 0 ? p.part_cols : D;
  float* part = p.part + size_t(blockIdx.x) * pc;
  for (int c = threadIdx.x; c < D; c += 256) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) s += red[k][c];
    part[c] = s;
  }
  if (has_b) {
    for (int c = threadIdx.x; c < p.H * D; c += 256) {
      const int h = c / D, d = c % D;
      float s = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if ((blockIdx.x * 8 + k) % p.H == h) s += red_b[k][d];
      part[D + c] = s;
    }
  }
}

// Fixed-order sums of the short-conv partial rows into dw [C, W] and dbias [C].
__global__ void __launch_bounds__(256) conv_param_sum_kernel(const float* part, int rows, int C,
                                                             int W, float* dw, float* dbias) {
  const int cols = C * (W + 1);
  const int idx = blockIdx.x * 256 + threadIdx.x;
  if (idx >= cols) return;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  int r = 0;
  for (; r + 4 <= rows; r += 4) {
    s0 += part[size_t(r) * cols + idx];
    s1 += part[size_t(r + 1) * cols + idx];
    s2 += part[size_t(r + 2) * cols + idx];
    s3 += part[size_t(r + 3) * cols + idx];
  }
  for (; r < rows; ++r) s0 += part[size_t(r) * cols + idx];
  const float s = (s0 + s1) + (s2 + s3);
  const int c = idx / (W + 1), i = idx % (W + 1);
  if (i < W)
    dw[c * W + i] = s;
  else if (dbias)
    dbias[c] = s;
}

// out[c] = sum_r part[r * row_stride + c] for c < cols (small cols), fixed order:
// 1024 threads split the rows, then a fixed-order tree over the threads.
__global__ void __launch_bounds__(1024) strided_column_sum_kernel(const float* part, float* out,
                                                                  int rows, int cols,
                                                                  int row_stride) {
  __shared__ float red[1024];
  for (int c = 0; c < cols; ++c) {
    float s = 0.f;
    for (int r = threadIdx.x; r < rows; r += 1024) s += part[size_t(r) * row_stride + c];
    red[threadIdx.x] = s;
    __syncthreads();
    for (int w = 512; w > 0; w >>= 1) {
      if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
      __syncthreads();
    }
    if (threadIdx.x == 0) out[c] = red[0];
    __syncthreads();
  }
}

// The four gate-parameter gradients from the [rows, 4H] partials of
// gate_act_bwd_kernel (dA_log | ddt_bias | db_bias | dd_bias), fixed order.
__global__ void __launch_bounds__(1024) gate_param_sum_kernel(const float* part, int rows, int H,
                                                              float* dA, float* ddt, float* dbb,
                                                              float* ddb) {
  // one warp per column; lanes stride the rows, then a fixed shuffle tree
  float* outs[4] = {dA, ddt, dbb, ddb};
  const int lane = threadIdx.x & 31;
  for (int c = threadIdx.x >> 5; c < 4 * H; c += 32) {
    float s = 0.f;
    for (int r = lane; r < rows; r += 32) s += part[size_t(r) * 4 * H + c];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0 && outs[c / H]) outs[c / H][c % H] = s;
  }
}

}  // namespace cyfa
