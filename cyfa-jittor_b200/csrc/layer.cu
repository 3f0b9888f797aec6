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

// Streaming short convolution: no shared-memory staging.  A warp walks a run of
// kConvRun consecutive tokens for a block of channels, keeping the W-1 previous
// input rows (packed bf16) in registers; each step issues the loads of
// kConvUnroll rows before any arithmetic, so every warp has several 256- or
// 512-byte row segments in flight.
constexpr int kConvRun = 32;     // tokens per warp
constexpr int kConvUnroll = 4;   // rows loaded ahead per step
constexpr int kConvWarps = 8;    // warps per CTA (consecutive token runs)

__device__ __forceinline__ float bf_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }

// Forward: lane owns channels c0 .. c0+3 (c0 = 128 * blockIdx.x + 4 * lane), and
// each step loads kConvUnrollF rows ahead.  y[t] = bias + sum_i w_i x[t - (W-1) + i];
// rows before t = 0 come from the cache (or are zero).
// grid (ceil(C/128), ceil(T / (kConvWarps*kConvRun)), B).
constexpr int kConvUnrollF = 8;

template <int W>
__global__ void __launch_bounds__(256) short_conv_fwd_kernel(ConvParams p) {
  pdl_wait();
  pdl_trigger();
  constexpr int WM = W > 1 ? W - 1 : 1;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int c0 = blockIdx.x * 128 + lane * 4, b = blockIdx.z;
  const int t0 = (blockIdx.y * kConvWarps + wid) * kConvRun;
  if (c0 >= p.C || t0 >= p.T) return;
  float wr[W][4], bias[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
#pragma unroll
    for (int i = 0; i < W; ++i) wr[i][e] = p.w[size_t(c0 + e) * W + i];
    bias[e] = p.bias ? p.bias[c0 + e] : 0.f;
  }
  const __nv_bfloat16* xb = p.x + size_t(b) * p.T * p.x_stride + c0;
  float win[WM][4];  // x rows t-(W-1) .. t-1, fp32
#pragma unroll
  for (int i = 0; i < W - 1; ++i) {
    const int t = t0 - (W - 1) + i;
    uint2 r = make_uint2(0, 0);
    if (t >= 0)
      r = *reinterpret_cast<const uint2*>(xb + size_t(t) * p.x_stride);
    else if (p.cache)
      r = *reinterpret_cast<const uint2*>(p.cache + (size_t(b) * (W - 1) + (W - 1) + t) * p.C + c0);
    win[i][0] = bf_lo(r.x), win[i][1] = bf_hi(r.x), win[i][2] = bf_lo(r.y), win[i][3] = bf_hi(r.y);
  }
  __nv_bfloat16* yb = p.y + size_t(b) * p.T * p.C + c0;
  const int tend = min(p.T, t0 + kConvRun);
  for (int t1 = t0; t1 < tend; t1 += kConvUnrollF) {
    uint2 cur[kConvUnrollF];
    const __nv_bfloat16* xr = xb + size_t(t1) * p.x_stride;
    if (t1 + kConvUnrollF <= tend) {
#pragma unroll
      for (int u = 0; u < kConvUnrollF; ++u)
        cur[u] = *reinterpret_cast<const uint2*>(xr + size_t(u) * p.x_stride);
    } else {
#pragma unroll
      for (int u = 0; u < kConvUnrollF; ++u)
        cur[u] = t1 + u < tend ? *reinterpret_cast<const uint2*>(xr + size_t(u) * p.x_stride)
                               : make_uint2(0, 0);
    }
#pragma unroll
    for (int u = 0; u < kConvUnrollF; ++u) {
      if (t1 + u >= tend) break;
      const float xn[4] = {bf_lo(cur[u].x), bf_hi(cur[u].x), bf_lo(cur[u].y), bf_hi(cur[u].y)};
      float y[4] = {bias[0], bias[1], bias[2], bias[3]};
#pragma unroll
      for (int i = 0; i < W; ++i) {
        const float* r = i < W - 1 ? win[i < W - 1 ? i : 0] : xn;
#pragma unroll
        for (int e = 0; e < 4; ++e) y[e] += wr[i][e] * r[e];
      }
      *reinterpret_cast<uint2*>(yb + size_t(t1 + u) * p.C) =
          make_uint2(pack_bf16(y[0], y[1]), pack_bf16(y[2], y[3]));
#pragma unroll
      for (int i = 0; i + 1 < W - 1; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) win[i][e] = win[i + 1][e];
      if (W > 1) {
#pragma unroll
        for (int e = 0; e < 4; ++e) win[W > 1 ? W - 2 : 0][e] = xn[e];
      }
    }
  }
}

// Backward without cache, lane owns channels c0 .. c0+3 (c0 = 128 * blockIdx.x + 4 * lane):
//   dx[t] = sum_i w_i dy[t + (W-1) - i],  dw_i = sum_t dy[t] x[t + i - (W-1)],
//   dbias = sum_t dy[t].
// A warp keeps x rows t-(W-1) .. t-1 and dy rows t .. t+W-2 in registers, unpacked
// once to fp32 as they arrive; each step loads kConvUnroll rows of both ahead
// (bounds checks only on the last step of a batch row).  The 8 warps of a CTA
// (consecutive token runs of one batch row) add their dw/dbias sums in a fixed
// order into one partial row per CTA row index blockIdx.y.
// grid (ceil(C/128), B * ceil(T / (kConvWarps*kConvRun))).
__device__ __forceinline__ void unpack4(uint2 r, float* f) {
  f[0] = bf_lo(r.x), f[1] = bf_hi(r.x), f[2] = bf_lo(r.y), f[3] = bf_hi(r.y);
}

template <int W>
__global__ void __launch_bounds__(256, 2) short_conv_bwd_kernel(ConvParams p) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[kConvWarps][128 * (W + 1)];
  constexpr int WM = W > 1 ? W - 1 : 1;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int ng = (p.T + kConvWarps * kConvRun - 1) / (kConvWarps * kConvRun);
  const int b = blockIdx.y / ng, grp = blockIdx.y % ng;
  const int c0 = blockIdx.x * 128 + lane * 4;
  const int t0 = (grp * kConvWarps + wid) * kConvRun;
  float acc[W + 1][4];
#pragma unroll
  for (int i = 0; i <= W; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[i][e] = 0.f;
  if (c0 < p.C && t0 < p.T) {
    float wr[W][4];
#pragma unroll
    for (int e = 0; e < 4; ++e)
#pragma unroll
      for (int i = 0; i < W; ++i) wr[i][e] = p.w[size_t(c0 + e) * W + i];
    const __nv_bfloat16* xb = p.x + size_t(b) * p.T * p.x_stride + c0;
    const __nv_bfloat16* db = p.dy + size_t(b) * p.T * p.C + c0;
    __nv_bfloat16* dxb = p.dx + size_t(b) * p.T * p.dx_stride + c0;
    float X[WM][4], D[WM][4];
#pragma unroll
    for (int i = 0; i < W - 1; ++i) {
      const int tx = t0 - (W - 1) + i, td = t0 + i;
      unpack4(tx >= 0 ? *reinterpret_cast<const uint2*>(xb + size_t(tx) * p.x_stride)
                      : make_uint2(0, 0), X[i]);
      unpack4(td < p.T ? *reinterpret_cast<const uint2*>(db + size_t(td) * p.C) : make_uint2(0, 0),
              D[i]);
    }
    const int tend = min(p.T, t0 + kConvRun);
    for (int t1 = t0; t1 < tend; t1 += kConvUnroll) {
      uint2 xs[kConvUnroll], ds[kConvUnroll];
      const __nv_bfloat16* xr = xb + size_t(t1) * p.x_stride;
      const __nv_bfloat16* dr = db + size_t(t1 + W - 1) * p.C;
      if (t1 + kConvUnroll <= tend && t1 + kConvUnroll + W - 1 <= p.T) {
#pragma unroll
        for (int u = 0; u < kConvUnroll; ++u) {
          xs[u] = *reinterpret_cast<const uint2*>(xr + size_t(u) * p.x_stride);
          ds[u] = *reinterpret_cast<const uint2*>(dr + size_t(u) * p.C);
        }
      } else {
#pragma unroll
        for (int u = 0; u < kConvUnroll; ++u) {
          const int t = t1 + u, td = t + W - 1;
          xs[u] = t < tend ? *reinterpret_cast<const uint2*>(xr + size_t(u) * p.x_stride)
                           : make_uint2(0, 0);
          ds[u] = (t < tend && td < p.T) ? *reinterpret_cast<const uint2*>(dr + size_t(u) * p.C)
                                         : make_uint2(0, 0);
        }
      }
#pragma unroll
      for (int u = 0; u < kConvUnroll; ++u) {
        if (t1 + u >= tend) break;
        float xn[4], dn[4];
        unpack4(xs[u], xn);
        unpack4(ds[u], dn);
        // dy rows t .. t+W-1 = D[0..W-2], dn;  x rows t-(W-1) .. t = X[0..W-2], xn
        float dx[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < W; ++i) {
          const int j = W - 1 - i;  // dy row t + j
          const float* dv = j < W - 1 ? D[j < W - 1 ? j : 0] : dn;
          const float* xv = i < W - 1 ? X[i < W - 1 ? i : 0] : xn;
          const float* d0 = W > 1 ? D[0] : dn;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            dx[e] += wr[i][e] * dv[e];
            acc[i][e] += d0[e] * xv[e];
          }
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[W][e] += (W > 1 ? D[0] : dn)[e];
        *reinterpret_cast<uint2*>(dxb + size_t(t1 + u) * p.dx_stride) =
            make_uint2(pack_bf16(dx[0], dx[1]), pack_bf16(dx[2], dx[3]));
#pragma unroll
        for (int i = 0; i + 1 < W - 1; ++i)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            X[i][e] = X[i + 1][e];
            D[i][e] = D[i + 1][e];
          }
        if (W > 1) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            X[W > 1 ? W - 2 : 0][e] = xn[e];
            D[W > 1 ? W - 2 : 0][e] = dn[e];
          }
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i <= W; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) red[wid][(lane * 4 + e) * (W + 1) + i] = acc[i][e];
  __syncthreads();
  for (int idx = threadIdx.x; idx < 128 * (W + 1); idx += 256) {
    const int c = blockIdx.x * 128 + idx / (W + 1);
    if (c >= p.C) continue;
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < kConvWarps; ++k) sum += red[k][idx];
    p.part[size_t(blockIdx.y) * (size_t(p.C) * (W + 1)) + size_t(c) * (W + 1) + idx % (W + 1)] =
        sum;
  }
}

// Partial rows of the backward for a shape.
inline int conv_bwd_rows(int B, int T) {
  return B * ((T + kConvWarps * kConvRun - 1) / (kConvWarps * kConvRun));
}

// ------------------------------------------------ TMA-streamed short convolution
// Without a conv cache and with C % 128 == 0 the convolution streams tiles of
// kCtRows tokens x 128 channels of one batch row through a shared-memory ring:
// warp 8 (one lane) issues 3-D TMA loads of the tile and its kCtHalo rows of
// context (x rows t0-3 .. t0+63, dy rows t0 .. t0+66; rows outside [0, T) read
// as zeros), warps 0-7 compute 8 tokens each from shared memory (lane = 4
// channels, sliding register window) and store their rows directly.  The CTAs
// are persistent, so the loads of the next tiles overlap the current one, and
// two share an SM (rings of 69 KiB), so one's loads also overlap the other's
// arithmetic.
constexpr int kCtRows = 64;
constexpr int kCtHalo = 3;                           // context rows (W <= 4)
constexpr int kCtBoxRows = kCtRows + kCtHalo;        // 67
constexpr int kCtTileBytes = kCtBoxRows * 128 * 2;   // 17152 (a multiple of 128)
constexpr int kCtStages = 4;                         // forward: x tiles
constexpr int kCtStagesB = 2;                        // backward: x and dy tiles
constexpr int kCtSmem = kCtStages * kCtTileBytes + 1024;
constexpr int kCtSmemB = kCtStagesB * 2 * kCtTileBytes + 1024;
static_assert(kCtSmem <= 227 * 1024 && kCtSmemB <= 227 * 1024, "conv ring");

struct ConvTmaParams {
  int B, T, C, nT;               // nT = tiles per batch row
  const float* w;                // [C, W]
  const float* bias;             // [C] or null (forward)
  __nv_bfloat16* out;            // forward y [B,T,C] dense; backward dx (token stride out_stride)
  long long out_stride;
  float* part;                   // backward: [G, C * (W + 1)] partial dw | dbias
};

__device__ __forceinline__ void ld_row4(const uint8_t* tile, int row, int lane, float* f) {
  const uint2 r = *reinterpret_cast<const uint2*>(tile + row * 256 + lane * 8);
  f[0] = __uint_as_float(r.x << 16), f[1] = __uint_as_float(r.x & 0xffff0000u);
  f[2] = __uint_as_float(r.y << 16), f[3] = __uint_as_float(r.y & 0xffff0000u);
}

// Forward: CTA (cb, g) = (blockIdx.x % ncb, blockIdx.x / ncb) owns channel block cb
// (its weights stay in registers) and the token tiles g, g + G, ... (G = gridDim.x
// / ncb) of all batch rows.  y[t] = bias + sum_i w_i x[t - (W-1) + i].
template <int W>
__global__ void __launch_bounds__(288, 1)
    short_conv_fwd_tma_kernel(const __grid_constant__ CUtensorMap map_x, ConvTmaParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[kCtStages], empty[kCtStages];
  __shared__ int s_abort;
  volatile int* abort_flag = &s_abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ncb = p.C / 128, G = gridDim.x / ncb;
  const int cb = blockIdx.x % ncb, g = blockIdx.x / ncb;
  const int ntiles = g < G ? p.B * p.nT : 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kCtStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 8);
    }
    s_abort = 0;
    mbar_fence_init();
    prefetch_tmap(&map_x);
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();
  if (warp == 8) {
    if (lane == 0) {
      int issued = 0;
      for (int i = 0, k = g; k < ntiles; ++i, k += G) {
        const int s = i % kCtStages;
        if (i >= kCtStages && !mbar_wait(&empty[s], ((i / kCtStages) - 1) & 1)) {
          *abort_flag = 1;
          break;
        }
        const int b = k / p.nT, t0 = (k % p.nT) * kCtRows;
        mbar_expect_tx(&full[s], kCtTileBytes);
        tma_load_3d(smem + s * kCtTileBytes, &map_x, &full[s], cb * 128, t0 - kCtHalo, b);
        issued = i + 1;
      }
      for (int i = issued > kCtStages ? issued - kCtStages : 0; i < issued; ++i)
        mbar_wait(&full[i % kCtStages], (i / kCtStages) & 1);
    }
    return;
  }
  const int c0 = cb * 128 + lane * 4;
  float wr[W][4], bias[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
#pragma unroll
    for (int q = 0; q < W; ++q) wr[q][e] = p.w[size_t(c0 + e) * W + q];
    bias[e] = p.bias ? p.bias[c0 + e] : 0.f;
  }
  for (int i = 0, k = g; k < ntiles; ++i, k += G) {
    const int s = i % kCtStages;
    const bool got = __all_sync(0xffffffffu, *abort_flag == 0 &&
                                                 mbar_wait(&full[s], (i / kCtStages) & 1));
    if (!got) {
      *abort_flag = 1;
      break;
    }
    const int b = k / p.nT, t0 = (k % p.nT) * kCtRows;
    const uint8_t* tile = smem + s * kCtTileBytes;
    const int r0 = warp * 8;  // first token row of this warp in the tile
    float win[W > 1 ? W - 1 : 1][4];
#pragma unroll
    for (int q = 0; q < W - 1; ++q) ld_row4(tile, r0 + kCtHalo - (W - 1) + q, lane, win[q]);
    __nv_bfloat16* yb = p.out + (size_t(b) * p.T + t0 + r0) * p.C + c0;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      float xn[4];
      ld_row4(tile, r0 + kCtHalo + u, lane, xn);
      float y[4] = {bias[0], bias[1], bias[2], bias[3]};
#pragma unroll
      for (int q = 0; q < W; ++q) {
        const float* r = q < W - 1 ? win[q < W - 1 ? q : 0] : xn;
#pragma unroll
        for (int e = 0; e < 4; ++e) y[e] += wr[q][e] * r[e];
      }
      if (t0 + r0 + u < p.T)
        *reinterpret_cast<uint2*>(yb + size_t(u) * p.C) =
            make_uint2(pack_bf16(y[0], y[1]), pack_bf16(y[2], y[3]));
#pragma unroll
      for (int q = 0; q + 1 < W - 1; ++q)
#pragma unroll
        for (int e = 0; e < 4; ++e) win[q][e] = win[q + 1][e];
      if (W > 1) {
#pragma unroll
        for (int e = 0; e < 4; ++e) win[W > 1 ? W - 2 : 0][e] = xn[e];
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
}

// Backward: CTA (cb, g) = (blockIdx.x % ncb, blockIdx.x / ncb) owns channel block
// cb and the token tiles g, g + G, ... (G = gridDim.x / ncb) of all batch rows, so
// its dw / dbias sums (registers, then a fixed-order block reduction) form one
// partial row g.  dx[t] = sum_i w_i dy[t + (W-1) - i], dw_i = sum_t dy[t] x[t + i - (W-1)].
template <int W>
__global__ void __launch_bounds__(288, 2)
    short_conv_bwd_tma_kernel(const __grid_constant__ CUtensorMap map_x,
                              const __grid_constant__ CUtensorMap map_dy, ConvTmaParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[kCtStagesB], empty[kCtStagesB];
  __shared__ int s_abort;
  __shared__ float red[8][128 * (W + 1)];
  volatile int* abort_flag = &s_abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ncb = p.C / 128, G = gridDim.x / ncb;
  const int cb = blockIdx.x % ncb, g = blockIdx.x / ncb;
  const int ntiles = p.B * p.nT;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kCtStagesB; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 8);
    }
    s_abort = 0;
    mbar_fence_init();
    prefetch_tmap(&map_x);
    prefetch_tmap(&map_dy);
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();
  float acc[W + 1][4];
#pragma unroll
  for (int q = 0; q <= W; ++q)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[q][e] = 0.f;
  if (warp == 8) {
    if (lane == 0 && g < G) {
      int issued = 0;
      for (int i = 0, k = g; k < ntiles; ++i, k += G) {
        const int s = i % kCtStagesB;
        if (i >= kCtStagesB && !mbar_wait(&empty[s], ((i / kCtStagesB) - 1) & 1)) {
          *abort_flag = 1;
          break;
        }
        const int b = k / p.nT, t0 = (k % p.nT) * kCtRows;
        uint8_t* st = smem + s * 2 * kCtTileBytes;
        mbar_expect_tx(&full[s], 2 * kCtTileBytes);
        tma_load_3d(st, &map_x, &full[s], cb * 128, t0 - kCtHalo, b);
        tma_load_3d(st + kCtTileBytes, &map_dy, &full[s], cb * 128, t0, b);
        issued = i + 1;
      }
      for (int i = issued > kCtStagesB ? issued - kCtStagesB : 0; i < issued; ++i)
        mbar_wait(&full[i % kCtStagesB], (i / kCtStagesB) & 1);
    }
  } else if (g < G) {
    const int c0 = cb * 128 + lane * 4;
    float wr[W][4];
#pragma unroll
    for (int e = 0; e < 4; ++e)
#pragma unroll
      for (int q = 0; q < W; ++q) wr[q][e] = p.w[size_t(c0 + e) * W + q];
    constexpr int WM = W > 1 ? W - 1 : 1;
    for (int i = 0, k = g; k < ntiles; ++i, k += G) {
      const int s = i % kCtStagesB;
      const bool got = __all_sync(0xffffffffu, *abort_flag == 0 &&
                                                   mbar_wait(&full[s], (i / kCtStagesB) & 1));
      if (!got) {
        *abort_flag = 1;
        break;
      }
      const int b = k / p.nT, t0 = (k % p.nT) * kCtRows;
      const uint8_t* xt = smem + s * 2 * kCtTileBytes;
      const uint8_t* dt = xt + kCtTileBytes;
      const int r0 = warp * 8;
      // x rows t-(W-1) .. t-1 and dy rows t .. t+W-2 of the warp's first token t
      float X[WM][4], D[WM][4];
#pragma unroll
      for (int q = 0; q < W - 1; ++q) {
        ld_row4(xt, r0 + kCtHalo - (W - 1) + q, lane, X[q]);
        ld_row4(dt, r0 + q, lane, D[q]);
      }
      __nv_bfloat16* dxb = p.out + (size_t(b) * p.T + t0 + r0) * p.out_stride + c0;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        float xn[4], dn[4];
        ld_row4(xt, r0 + kCtHalo + u, lane, xn);  // x[t]
        ld_row4(dt, r0 + u + W - 1, lane, dn);    // dy[t + W - 1]
        const float* d0 = W > 1 ? D[0] : dn;      // dy[t]
        float dx[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int q = 0; q < W; ++q) {
          const int j = W - 1 - q;  // dy row t + j
          const float* dv = j < W - 1 ? D[j < W - 1 ? j : 0] : dn;
          const float* xv = q < W - 1 ? X[q < W - 1 ? q : 0] : xn;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            dx[e] += wr[q][e] * dv[e];
            acc[q][e] += d0[e] * xv[e];
          }
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[W][e] += d0[e];
        if (t0 + r0 + u < p.T)
          *reinterpret_cast<uint2*>(dxb + size_t(u) * p.out_stride) =
              make_uint2(pack_bf16(dx[0], dx[1]), pack_bf16(dx[2], dx[3]));
#pragma unroll
        for (int q = 0; q + 1 < W - 1; ++q)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            X[q][e] = X[q + 1][e];
            D[q][e] = D[q + 1][e];
          }
        if (W > 1) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            X[W > 1 ? W - 2 : 0][e] = xn[e];
            D[W > 1 ? W - 2 : 0][e] = dn[e];
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
  }
  if (warp < 8) {
#pragma unroll
    for (int q = 0; q <= W; ++q)
#pragma unroll
      for (int e = 0; e < 4; ++e) red[warp][(lane * 4 + e) * (W + 1) + q] = acc[q][e];
  }
  __syncthreads();
  if (g >= G) return;
  for (int idx = threadIdx.x; idx < 128 * (W + 1); idx += blockDim.x) {
    float sum = 0.f;
#pragma unroll
    for (int w8 = 0; w8 < 8; ++w8) sum += red[w8][idx];
    p.part[size_t(g) * (size_t(p.C) * (W + 1)) + size_t(cb) * 128 * (W + 1) + idx] = sum;
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
// Sigmoid from the fast exponential and division intrinsics (a few ulp), for the
// gated norm whose outputs are rounded to bf16.
__device__ __forceinline__ float sigmoid_fast(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }

__global__ void __launch_bounds__(256) gate_act_fwd_kernel(GateActParams p) {
  pdl_wait();
  pdl_trigger();
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
  pdl_wait();
  pdl_trigger();
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

// One warp per row, grid-strided, two rows per iteration (loads of both rows
// issued first).  The weight (and, with a gate bias, the bias of the warp's head:
// the grid is then a multiple of H, so (blockIdx.x * 8 + warp) % H is the head of
// every row the warp visits) stays in registers.  D = 32 * E.
template <int E>
__global__ void __launch_bounds__(256, 3) gated_norm_fwd_kernel(GatedNormParams p) {
  pdl_wait();
  pdl_trigger();
  constexpr int D = 32 * E;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const size_t stride = size_t(gridDim.x) * 8;
  float w[E], bias[E];
  load_f32_vec<E>(p.w + lane * E, w);
#pragma unroll
  for (int e = 0; e < E; ++e) bias[e] = 0.f;
  if (p.gbias) load_bf16_vec<E>(p.gbias + size_t((blockIdx.x * 8 + wid) % p.H) * D + lane * E, bias);
  for (size_t row0 = size_t(blockIdx.x) * 8 + wid; row0 < size_t(p.rows); row0 += 2 * stride) {
    float x[2][E], g[2][E];
    bool live[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const size_t row = row0 + u * stride;
      live[u] = row < size_t(p.rows);
      if (live[u]) {
        load_bf16_vec<E>(p.x + row * D + lane * E, x[u]);
        load_bf16_vec<E>(p.gate + row * D + lane * E, g[u]);
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) x[u][e] = g[u][e] = 0.f;
      }
    }
    // both rows' reductions interleaved (independent shuffle chains)
    float ss[2] = {0.f, 0.f};
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
      for (int e = 0; e < E; ++e) {
        x[u][e] *= p.scale;
        ss[u] += x[u][e] * x[u][e];
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ss[0] += __shfl_xor_sync(0xffffffffu, ss[0], o);
      ss[1] += __shfl_xor_sync(0xffffffffu, ss[1], o);
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      if (!live[u]) continue;
      const size_t row = row0 + u * stride;
      const float rs = rsqrtf(ss[u] / D + p.eps);
      if (lane == 0) p.rstd[row] = rs;
      float y[E];
#pragma unroll
      for (int e = 0; e < E; ++e) y[e] = x[u][e] * rs * w[e] * sigmoid_fast(g[u][e] + bias[e]);
      store_bf16_vec<E>(p.y + row * D + lane * E, y);
    }
  }
}

// Grid of the gated-norm forward: two rows per warp per pass, three blocks per SM,
// a multiple of H (see above).
inline int norm_fwd_blocks(int rows, int H) {
  int n = (rows + 15) / 16;
  if (n > 444) n = 444;
  n -= n % H;
  return n < H ? H : n;
}

// Same warp/head rule as the forward.  Register-lean: n, dn and dgate overwrite
// x, dy and the gate in place.
template <int E>
__global__ void __launch_bounds__(256, 3) gated_norm_bwd_kernel(GatedNormParams p) {
  pdl_wait();
  pdl_trigger();
  constexpr int D = 32 * E;
  __shared__ float red[8][D];
  __shared__ float red_b[8][D];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const bool has_b = p.gbias != nullptr;
  float w[E], acc[E], acc_b[E], bias[E];
  load_f32_vec<E>(p.w + lane * E, w);
#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] = acc_b[e] = bias[e] = 0.f;
  if (has_b) load_bf16_vec<E>(p.gbias + size_t((blockIdx.x * 8 + wid) % p.H) * D + lane * E, bias);
  for (int row = blockIdx.x * 8 + wid; row < p.rows; row += gridDim.x * 8) {
    float x[E], g[E], dy[E];
    load_bf16_vec<E>(p.x + size_t(row) * D + lane * E, x);
    load_bf16_vec<E>(p.gate + size_t(row) * D + lane * E, g);
    load_bf16_vec<E>(p.dy + size_t(row) * D + lane * E, dy);
    const float rs = p.rstd[row];
    float dot = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float sg = sigmoid_fast(g[e] + bias[e]);
      const float n = x[e] * p.scale * rs;
      const float dz = dy[e] * sg;
      g[e] = dy[e] * n * w[e] * sg * (1.f - sg);  // dgate
      acc[e] += dz * n;
      acc_b[e] += g[e];
      dy[e] = dz * w[e];  // dn
      x[e] = n;
      dot += dy[e] * n;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    dot /= D;
#pragma unroll
    for (int e = 0; e < E; ++e) dy[e] = p.scale * rs * (dy[e] - x[e] * dot);  // dx
    store_bf16_vec<E>(p.dx + size_t(row) * D + lane * E, dy);
    store_bf16_vec<E>(p.dgate + size_t(row) * D + lane * E, g);
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

// TMA-streamed forward of the biased gated norm: the tile scheme of the backward
// below (CTA = head x token-tile group, warp 8 loads x and gate tiles, warps 0-7
// four tokens each), y and rstd stored directly; a 3-stage ring (97 KiB), two
// CTAs per SM.
constexpr int kNtRows = 32;
constexpr int kNtStagesF = 3;

template <int E>
constexpr int norm_fwd_tma_smem() {
  return kNtStagesF * 2 * kNtRows * 32 * E * 2 + 1024;
}

template <int E>
__global__ void __launch_bounds__(288, 1)
    gated_norm_fwd_tma_kernel(const __grid_constant__ CUtensorMap map_x,
                              const __grid_constant__ CUtensorMap map_g, GatedNormParams p) {
  constexpr int D = 32 * E, LB = 2 * E;
  constexpr int kTile = kNtRows * D * 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[kNtStagesF], empty[kNtStagesF];
  __shared__ int s_abort;
  volatile int* abort_flag = &s_abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = p.H, G = gridDim.x / H, h = blockIdx.x % H, g = blockIdx.x / H;
  const int BT = p.rows / H, ntiles = g < G ? (BT + kNtRows - 1) / kNtRows : 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kNtStagesF; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 8);
    }
    s_abort = 0;
    mbar_fence_init();
    prefetch_tmap(&map_x);
    prefetch_tmap(&map_g);
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();
  if (warp == 8) {
    if (lane == 0) {
      int issued = 0;
      for (int i = 0, tb = g; tb < ntiles; ++i, tb += G) {
        const int s = i % kNtStagesF;
        if (i >= kNtStagesF && !mbar_wait(&empty[s], ((i / kNtStagesF) - 1) & 1)) {
          *abort_flag = 1;
          break;
        }
        uint8_t* st = smem + s * 2 * kTile;
        mbar_expect_tx(&full[s], 2 * kTile);
        tma_load_3d(st, &map_x, &full[s], 0, h, tb * kNtRows);
        tma_load_3d(st + kTile, &map_g, &full[s], 0, h, tb * kNtRows);
        issued = i + 1;
      }
      for (int i = issued > kNtStagesF ? issued - kNtStagesF : 0; i < issued; ++i)
        mbar_wait(&full[i % kNtStagesF], (i / kNtStagesF) & 1);
    }
    return;
  }
  float w[E], bias[E];
  load_f32_vec<E>(p.w + lane * E, w);
  if (p.gbias) {
    load_bf16_vec<E>(p.gbias + size_t(h) * D + lane * E, bias);
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e) bias[e] = 0.f;
  }
  const int r0 = warp * 4;
  for (int i = 0, tb = g; tb < ntiles; ++i, tb += G) {
    const int s = i % kNtStagesF;
    const bool got = __all_sync(0xffffffffu, *abort_flag == 0 &&
                                                 mbar_wait(&full[s], (i / kNtStagesF) & 1));
    if (!got) {
      *abort_flag = 1;
      break;
    }
    const uint8_t* st = smem + s * 2 * kTile;
    // the four rows' reductions interleaved
    float x[4][E], ss[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      load_bf16_vec<E>(reinterpret_cast<const __nv_bfloat16*>(st + (r0 + u) * D * 2 + lane * LB),
                       x[u]);
      ss[u] = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        x[u][e] *= p.scale;
        ss[u] += x[u][e] * x[u][e];
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int u = 0; u < 4; ++u) ss[u] += __shfl_xor_sync(0xffffffffu, ss[u], o);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int tok = tb * kNtRows + r0 + u;
      float gt[E];
      load_bf16_vec<E>(
          reinterpret_cast<const __nv_bfloat16*>(st + kTile + (r0 + u) * D * 2 + lane * LB), gt);
      const float rs = rsqrtf(ss[u] / D + p.eps);
      float y[E];
#pragma unroll
      for (int e = 0; e < E; ++e) y[e] = x[u][e] * rs * w[e] * sigmoid_fast(gt[e] + bias[e]);
      if (tok < BT) {
        const size_t row = size_t(tok) * H + h;
        store_bf16_vec<E>(p.y + row * D + lane * E, y);
        if (lane == 0) p.rstd[row] = rs;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
}

// TMA-streamed backward of the biased gated norm.  CTA c owns head h = c % H and
// the 32-token tiles g, g + G, ... (g = c / H, G = gridDim.x / H) of that head:
// warp 8 (one lane) brings the tile's x, gate and dy rows ([32, D] each, 3-D maps
// {D, H, tokens}) into a shared ring, warps 0-7 take four tokens each.  The
// weight and the head's gate bias stay in registers, so the warp sums of the
// weight and gate-bias gradients need no per-row head bookkeeping.
constexpr int kNtStagesB = 4;

template <int E>
constexpr int norm_bwd_tma_smem() {
  return kNtStagesB * 3 * kNtRows * 32 * E * 2 + 1024;
}

template <int E>
__global__ void __launch_bounds__(288, 1)
    gated_norm_bwd_tma_kernel(const __grid_constant__ CUtensorMap map_x,
                              const __grid_constant__ CUtensorMap map_g,
                              const __grid_constant__ CUtensorMap map_dy, GatedNormParams p) {
  constexpr int D = 32 * E, LB = 2 * E;
  constexpr int kTile = kNtRows * D * 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[kNtStagesB], empty[kNtStagesB];
  __shared__ int s_abort;
  __shared__ float red[8][D];
  __shared__ float red_b[8][D];
  volatile int* abort_flag = &s_abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = p.H, G = gridDim.x / H, h = blockIdx.x % H, g = blockIdx.x / H;
  const int BT = p.rows / H, ntiles = g < G ? (BT + kNtRows - 1) / kNtRows : 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kNtStagesB; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 8);
    }
    s_abort = 0;
    mbar_fence_init();
    prefetch_tmap(&map_x);
    prefetch_tmap(&map_g);
    prefetch_tmap(&map_dy);
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();
  float acc[E], acc_b[E];
#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] = acc_b[e] = 0.f;
  if (warp == 8) {
    if (lane == 0) {
      int issued = 0;
      for (int i = 0, tb = g; tb < ntiles; ++i, tb += G) {
        const int s = i % kNtStagesB;
        if (i >= kNtStagesB && !mbar_wait(&empty[s], ((i / kNtStagesB) - 1) & 1)) {
          *abort_flag = 1;
          break;
        }
        uint8_t* st = smem + s * 3 * kTile;
        mbar_expect_tx(&full[s], 3 * kTile);
        tma_load_3d(st, &map_x, &full[s], 0, h, tb * kNtRows);
        tma_load_3d(st + kTile, &map_g, &full[s], 0, h, tb * kNtRows);
        tma_load_3d(st + 2 * kTile, &map_dy, &full[s], 0, h, tb * kNtRows);
        issued = i + 1;
      }
      for (int i = issued > kNtStagesB ? issued - kNtStagesB : 0; i < issued; ++i)
        mbar_wait(&full[i % kNtStagesB], (i / kNtStagesB) & 1);
    }
  } else {
    float w[E], bias[E];
    load_f32_vec<E>(p.w + lane * E, w);
    load_bf16_vec<E>(p.gbias + size_t(h) * D + lane * E, bias);
    const int r0 = warp * 4;
    // rstd of the warp's four rows, one tile ahead (lanes 0-3)
    auto rstd_of = [&](int tb) {
      const int tok = tb * kNtRows + r0 + lane;
      return (lane < 4 && tb < ntiles && tok < BT) ? p.rstd[size_t(tok) * H + h] : 0.f;
    };
    float rs_cur = rstd_of(g);
    for (int i = 0, tb = g; tb < ntiles; ++i, tb += G) {
      const float rs_next = rstd_of(tb + G);
      const int s = i % kNtStagesB;
      const bool got = __all_sync(0xffffffffu, *abort_flag == 0 &&
                                                   mbar_wait(&full[s], (i / kNtStagesB) & 1));
      if (!got) {
        *abort_flag = 1;
        break;
      }
      const uint8_t* st = smem + s * 3 * kTile;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int tok = tb * kNtRows + r0 + u;
        const float rs = __shfl_sync(0xffffffffu, rs_cur, u);
        float x[E], gt[E], dy[E];
        const int off = (r0 + u) * D * 2 + lane * LB;
        load_bf16_vec<E>(reinterpret_cast<const __nv_bfloat16*>(st + off), x);
        load_bf16_vec<E>(reinterpret_cast<const __nv_bfloat16*>(st + kTile + off), gt);
        load_bf16_vec<E>(reinterpret_cast<const __nv_bfloat16*>(st + 2 * kTile + off), dy);
        float dot = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const float sg = sigmoid_fast(gt[e] + bias[e]);
          const float n = x[e] * p.scale * rs;
          const float dz = dy[e] * sg;
          gt[e] = dy[e] * n * w[e] * sg * (1.f - sg);  // dgate
          dy[e] = dz * w[e];                           // dn
          x[e] = n;
          if (tok < BT) {
            acc[e] += dz * n;
            acc_b[e] += gt[e];
          }
          dot += dy[e] * n;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        dot /= D;
#pragma unroll
        for (int e = 0; e < E; ++e) dy[e] = p.scale * rs * (dy[e] - x[e] * dot);  // dx
        if (tok < BT) {
          const size_t row = size_t(tok) * H + h;
          store_bf16_vec<E>(p.dx + row * D + lane * E, dy);
          store_bf16_vec<E>(p.dgate + row * D + lane * E, gt);
        }
      }
      rs_cur = rs_next;
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
  }
  if (warp < 8) {
#pragma unroll
    for (int e = 0; e < E; ++e) {
      red[warp][lane * E + e] = acc[e];
      red_b[warp][lane * E + e] = acc_b[e];
    }
  }
  __syncthreads();
  const int pc = p.part_cols;
  float* part = p.part + size_t(blockIdx.x) * pc;
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float sw = 0.f, sb = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      sw += red[k][c];
      sb += red_b[k][c];
    }
    part[c] = sw;
    for (int hh = 0; hh < H; ++hh) part[D + hh * D + c] = hh == h ? sb : 0.f;
  }
}

// Fixed-order sums of the short-conv partial rows into dw [C, W] and dbias [C].
__global__ void __launch_bounds__(256) conv_param_sum_kernel(const float* part, int rows, int C,
                                                             int W, float* dw, float* dbias) {
  pdl_wait();
  pdl_trigger();
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
  pdl_wait();
  pdl_trigger();
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
  pdl_wait();
  pdl_trigger();
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
