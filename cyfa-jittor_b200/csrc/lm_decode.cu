// Decoder-block glue for one recurrent decode step of the CyFA language model.
//
// A decode step of the LM moves little data per kernel (batch x hidden rows), so
// the cost of the plain-PyTorch glue around the attention core is its number of
// launches.  These kernels fold each piece of glue into one launch:
//   add_rmsnorm  : residual add + RMSNorm of the decoder blocks
//                  (models/cyfa/modeling_cyfa.py:52-55, 64-69; RMSNorm layers/cyfa.py:62-135)
//   decode_conv  : the q, k and v short convolutions for one token with their
//                  W-1 cached rows, the caches shifted in place
//                  (ShortConvolution with a cache, layers/cyfa.py:144-181)
//   swiglu       : the gated MLP activation g sigmoid(g) u
//                  (GatedMLP.execute, models/cyfa/modeling_cyfa.py:22-27)
//   decode_layer : the attention layer's step between its two projections for
//                  one (sequence, head): convolutions, gate activations,
//                  recurrent step and gated output norm
//                  (layers/cyfa.py:299-357 at T = 1 with a cache)
// All three are HBM/latency bound: each element is read and written once with
// 16-byte vector accesses, fp32 arithmetic, bf16 rounding where the reference
// rounds.

struct AddNormParams {
  __nv_bfloat16* x;        // [rows, D] residual stream (updated in place when y != null)
  const __nv_bfloat16* y;  // [rows, D] branch output or null
  const float* w;          // [D]
  __nv_bfloat16* out;      // [rows, D]
  float eps;
  int rows, D;
};

// One 256-thread CTA per row; thread t owns columns 8t + 2048j (j < 4, so
// D <= 8192), held in registers between the sum of squares and the output.
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(AddNormParams p) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[8];
  const int row = blockIdx.x, t = threadIdx.x;
  __nv_bfloat16* xr = p.x + (size_t)row * p.D;
  __align__(16) __nv_bfloat16 v[4][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int d = t * 8 + j * 2048;
    if (d < p.D) {
      *reinterpret_cast<int4*>(v[j]) = *reinterpret_cast<const int4*>(xr + d);
      if (p.y) {
        __align__(16) __nv_bfloat16 u[8];
        *reinterpret_cast<int4*>(u) = *reinterpret_cast<const int4*>(p.y + (size_t)row * p.D + d);
#pragma unroll
        for (int i = 0; i < 8; ++i)
          v[j][i] = __float2bfloat16_rn(__bfloat162float(v[j][i]) + __bfloat162float(u[i]));
        *reinterpret_cast<int4*>(xr + d) = *reinterpret_cast<int4*>(v[j]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float f = __bfloat162float(v[j][i]);
        ss += f * f;
      }
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (t % 32 == 0) red[t / 32] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) tot += red[w];  // same order in every thread
  const float rs = rsqrtf(tot / p.D + p.eps);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int d = t * 8 + j * 2048;
    if (d < p.D) {
      const float4 w0 = *reinterpret_cast<const float4*>(p.w + d);
      const float4 w1 = *reinterpret_cast<const float4*>(p.w + d + 4);
      const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      __align__(16) __nv_bfloat16 o8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) o8[i] = __float2bfloat16_rn(__bfloat162float(v[j][i]) * rs * wv[i]);
      *reinterpret_cast<int4*>(p.out + (size_t)row * p.D + d) = *reinterpret_cast<int4*>(o8);
    }
  }
}

struct DecodeConvParams {
  const __nv_bfloat16* x;  // row b: q|k|v pre-convolution values at x + b * x_stride
  long long x_stride;
  __nv_bfloat16* cache[3];  // [B, W-1, C_i], oldest row first; shifted in place
  const float* w[3];        // [C_i, W]
  __nv_bfloat16* y[3];      // [B, C_i]
  int C[3];
  int B, W;
};

// One thread per (sequence, 8 channels) over the three convolutions.  Each thread
// owns its cache column, so the in-place shift needs no synchronisation.  The
// eight channels' W taps are 8W consecutive floats, read as float4.
template <int W>
__global__ void __launch_bounds__(256) decode_conv_kernel(DecodeConvParams p) {
  pdl_wait();
  pdl_trigger();
  const int groups = (p.C[0] + p.C[1] + p.C[2]) / 8;
  const long long i = (long long)blockIdx.x * 256 + threadIdx.x;
  if (i >= (long long)p.B * groups) return;
  const int b = int(i / groups);
  int c = int(i % groups) * 8;
  const int col = c;  // column in the packed q|k|v row
  int s = 0;
  if (c >= p.C[0]) { c -= p.C[0]; s = 1; }
  if (s == 1 && c >= p.C[1]) { c -= p.C[1]; s = 2; }
  // select the convolution's pointers without indexing the parameter arrays by
  // a runtime value (which would copy them to local memory in every thread)
  const int C = s == 0 ? p.C[0] : (s == 1 ? p.C[1] : p.C[2]);
  __nv_bfloat16* const cache_s = s == 0 ? p.cache[0] : (s == 1 ? p.cache[1] : p.cache[2]);
  const float* const w_s = s == 0 ? p.w[0] : (s == 1 ? p.w[1] : p.w[2]);
  __nv_bfloat16* const y_s = s == 0 ? p.y[0] : (s == 1 ? p.y[1] : p.y[2]);
  __align__(16) __nv_bfloat16 hist[W][8];  // W-1 cached rows, then the new token
  __nv_bfloat16* cache = cache_s + (size_t)b * (W - 1) * C + c;
#pragma unroll
  for (int r = 0; r < W - 1; ++r)
    *reinterpret_cast<int4*>(hist[r]) = *reinterpret_cast<const int4*>(cache + (size_t)r * C);
  *reinterpret_cast<int4*>(hist[W - 1]) =
      *reinterpret_cast<const int4*>(p.x + (size_t)b * p.x_stride + col);
  float w[8 * W];
  const float4* w4 = reinterpret_cast<const float4*>(w_s + (size_t)c * W);
#pragma unroll
  for (int q = 0; q < 2 * W; ++q) {
    const float4 f = w4[q];
    w[4 * q] = f.x;
    w[4 * q + 1] = f.y;
    w[4 * q + 2] = f.z;
    w[4 * q + 3] = f.w;
  }
  __align__(16) __nv_bfloat16 out[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float acc = __bfloat162float(hist[0][j]) * w[j * W];
#pragma unroll
    for (int r = 1; r < W; ++r) acc += __bfloat162float(hist[r][j]) * w[j * W + r];
    out[j] = __float2bfloat16_rn(acc);
  }
  *reinterpret_cast<int4*>(y_s + (size_t)b * C + c) = *reinterpret_cast<int4*>(out);
#pragma unroll
  for (int r = 0; r < W - 1; ++r)
    *reinterpret_cast<int4*>(cache + (size_t)r * C) = *reinterpret_cast<int4*>(hist[r + 1]);
}

struct SwigluParams {
  const __nv_bfloat16* gu;  // [rows, 2 * mid]: gate columns, then up columns
  __nv_bfloat16* out;       // [rows, mid]
  int rows, mid;
};

__global__ void __launch_bounds__(256) swiglu_kernel(SwigluParams p) {
  pdl_wait();
  pdl_trigger();
  const int groups = p.mid / 8;
  const long long i = (long long)blockIdx.x * 256 + threadIdx.x;
  if (i >= (long long)p.rows * groups) return;
  const long long r = i / groups;
  const int m = int(i % groups) * 8;
  __align__(16) __nv_bfloat16 g[8], u[8], o[8];
  *reinterpret_cast<int4*>(g) = *reinterpret_cast<const int4*>(p.gu + r * 2 * p.mid + m);
  *reinterpret_cast<int4*>(u) = *reinterpret_cast<const int4*>(p.gu + r * 2 * p.mid + p.mid + m);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float gf = __bfloat162float(g[j]);
    o[j] = __float2bfloat16_rn(gf * sigmoid_f(gf) * __bfloat162float(u[j]));
  }
  *reinterpret_cast<int4*>(p.out + r * p.mid + m) = *reinterpret_cast<int4*>(o);
}

// One decode step of the CyFA layer's core for one (sequence, head), from the
// packed projection row to the gated-norm output: the three short convolutions
// of the head's q, k and v channels with their cached rows (shifted in place),
// the gate activations (g, delta, beta), the recurrent step (decode_token), and
// the output gate's RMSNorm with its bias.  It replaces the decode_conv,
// gate_act_fwd, decode_step and gated_norm launches of a layer step with one;
// every value is rounded where those kernels round it (convolution outputs and
// the core output to bf16), so the result is the same up to the order of the
// norm's row sum.
struct DecodeLayerParams {
  const __nv_bfloat16* P;       // [B, P_stride]: q | k | v | g0 | a | b | d (+pad)
  long long P_stride;
  int a_col;                    // column of a; b at a_col + H, d at a_col + 2H
  __nv_bfloat16* cache[3];      // q, k, v histories [B, W-1, C_i], oldest row first
  const float* wconv[3];        // [C_i, W]
  const float* A_log;           // [H]
  const float* dt_bias;         // [H]
  const float* b_bias;          // [H] or null
  const float* d_bias;          // [H] or null
  const float* table;           // [H, 127, 128] fp32
  const float* q_norm_weight;   // [K]
  const float* k_norm_weight;   // [K]
  const float* hk_in;           // [B*H, K, 128] or null (zero state)
  const float* hv_in;           // [B*H, 128, V] or null
  const float* clock_in;        // [B*H] or null
  float* hk_out;
  float* hv_out;
  float* clock_out;
  const __nv_bfloat16* gate;    // [B, H*V] output gate before its bias
  const __nv_bfloat16* gate_bias;  // [H*V]
  const float* o_norm_weight;   // [V]
  __nv_bfloat16* y;             // [B, H*V]
  int B, H;
  float q_eps, k_eps, scale, o_eps, o_scale;
};

template <int K, int V, int W>
__global__ void __launch_bounds__(256) decode_layer_kernel(DecodeLayerParams p) {
  pdl_wait();
  pdl_trigger();
  constexpr int M = 128;
  const int tid = threadIdx.x;
  const int bh = blockIdx.x, b = bh / p.H, h = bh % p.H;
  __shared__ __align__(16) __nv_bfloat16 s_in[2 * K + V];  // q | k | v after the convolutions
  __shared__ __align__(16) __nv_bfloat16 s_out[V];
  __shared__ float s_gate[3];  // g, delta, beta
  __shared__ float red[8];
  const __nv_bfloat16* prow = p.P + size_t(b) * p.P_stride;
  // ---- short convolutions: one thread per 8 channels of the head
  for (int grp = tid; grp < (2 * K + V) / 8; grp += 256) {
    const int e0 = grp * 8;  // element of q | k | v of this head
    const int s = e0 < K ? 0 : (e0 < 2 * K ? 1 : 2);
    const int C = s == 2 ? p.H * V : p.H * K;
    const int c = s == 2 ? h * V + (e0 - 2 * K) : h * K + (e0 - s * K);  // channel in conv s
    const int col = (s == 0 ? 0 : (s == 1 ? p.H * K : 2 * p.H * K)) + c;  // column of P
    __nv_bfloat16* const cache_s = s == 0 ? p.cache[0] : (s == 1 ? p.cache[1] : p.cache[2]);
    const float* const w_s = s == 0 ? p.wconv[0] : (s == 1 ? p.wconv[1] : p.wconv[2]);
    __nv_bfloat16* cache = cache_s + size_t(b) * (W - 1) * C + c;
    __align__(16) __nv_bfloat16 hist[W][8];
#pragma unroll
    for (int r = 0; r < W - 1; ++r)
      *reinterpret_cast<int4*>(hist[r]) = *reinterpret_cast<const int4*>(cache + size_t(r) * C);
    *reinterpret_cast<int4*>(hist[W - 1]) = *reinterpret_cast<const int4*>(prow + col);
    // taps read per channel (few registers live beside the decode step's)
    const float* wc = w_s + size_t(c) * W;
    __align__(16) __nv_bfloat16 out[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float acc = __bfloat162float(hist[0][j]) * __ldg(wc + j * W);
#pragma unroll
      for (int r = 1; r < W; ++r) acc += __bfloat162float(hist[r][j]) * __ldg(wc + j * W + r);
      out[j] = __float2bfloat16_rn(acc);
    }
    *reinterpret_cast<int4*>(s_in + e0) = *reinterpret_cast<int4*>(out);
#pragma unroll
    for (int r = 0; r < W - 1; ++r)
      *reinterpret_cast<int4*>(cache + size_t(r) * C) = *reinterpret_cast<int4*>(hist[r + 1]);
  }
  // ---- gate activations (gate_act_fwd_kernel's arithmetic)
  if (tid == 0) {
    const float a = __bfloat162float(prow[p.a_col + h]) + p.dt_bias[h];
    s_gate[0] = -expf(p.A_log[h]) * softplus_f(a);
    s_gate[1] = sigmoid_f(__bfloat162float(prow[p.a_col + 2 * p.H + h]) +
                          (p.d_bias ? p.d_bias[h] : 0.f));
    s_gate[2] = sigmoid_f(__bfloat162float(prow[p.a_col + p.H + h]) +
                          (p.b_bias ? p.b_bias[h] : 0.f));
  }
  __syncthreads();
  TokenIO io;
  io.q = s_in;
  io.k = s_in + K;
  io.v = s_in + 2 * K;
  io.g = s_gate[0];
  io.beta = s_gate[2];
  io.lam = (p.clock_in ? p.clock_in[bh] : 0.f) + s_gate[1];
  io.hk_src = p.hk_in ? p.hk_in + size_t(bh) * K * M : nullptr;
  io.hv_src = p.hv_in ? p.hv_in + size_t(bh) * M * V : nullptr;
  io.hk_dst = p.hk_out + size_t(bh) * K * M;
  io.hv_dst = p.hv_out + size_t(bh) * M * V;
  io.clock_dst = p.clock_out + bh;
  io.out = s_out;
  decode_token<__nv_bfloat16, K, V, true>(io, p.table + size_t(h) * 127 * M, p.q_norm_weight,
                                          p.k_norm_weight, p.q_eps, p.k_eps, p.scale);
  // ---- output gate norm of the head's row (gated_norm_fwd's arithmetic)
  const float x = tid < V ? __bfloat162float(s_out[tid]) * p.o_scale : 0.f;
  const float ss = block_sum_256(x * x, red);
  if (tid < V) {
    const float rs = rsqrtf(ss / V + p.o_eps);
    const size_t i = size_t(bh) * V + tid;  // [B, H*V] row b, column h*V + tid
    const float z = __bfloat162float(p.gate[i]) + __bfloat162float(p.gate_bias[h * V + tid]);
    p.y[i] = __float2bfloat16_rn(x * rs * p.o_norm_weight[tid] * sigmoid_fast(z));
  }
}

extern "C" {

int cyfa_decode_layer(const cyfa_decode_layer_args* a, void* stream) {
  CYFA_REQUIRE(a, kNullPointer);
  const int K = a->K, V = a->V, W = a->W, H = a->H, B = a->B;
  CYFA_REQUIRE(a->P && a->cache_q && a->cache_k && a->cache_v && a->wconv_q && a->wconv_k &&
                   a->wconv_v && a->A_log && a->dt_bias && a->table && a->q_norm_weight &&
                   a->k_norm_weight && a->hk_out && a->hv_out && a->clock_out && a->gate &&
                   a->gate_bias && a->o_norm_weight && a->y,
               kNullPointer);
  CYFA_REQUIRE(B > 0 && H > 0 && (K == 128 || K == 256) && (V == 128 || V == 256) && W >= 2 &&
                   W <= 4 && a->P_stride % 8 == 0 &&
                   a->P_stride >= (long long)a->a_col + 3 * H && a->a_col >= 2 * H * K + H * V,
               kBadShape);
  CYFA_REQUIRE(aligned(a->P, 16) && aligned(a->cache_q, 16) && aligned(a->cache_k, 16) &&
                   aligned(a->cache_v, 16) && aligned(a->wconv_q, 16) && aligned(a->wconv_k, 16) &&
                   aligned(a->wconv_v, 16) && aligned(a->hk_out, 16) && aligned(a->hv_out, 16) &&
                   aligned(a->table, 16) && (!a->hk_in || aligned(a->hk_in, 16)) &&
                   (!a->hv_in || aligned(a->hv_in, 16)),
               kMisaligned);
  DecodeLayerParams p{static_cast<const __nv_bfloat16*>(a->P),
                      a->P_stride,
                      a->a_col,
                      {static_cast<__nv_bfloat16*>(a->cache_q),
                       static_cast<__nv_bfloat16*>(a->cache_k),
                       static_cast<__nv_bfloat16*>(a->cache_v)},
                      {a->wconv_q, a->wconv_k, a->wconv_v},
                      a->A_log,
                      a->dt_bias,
                      a->b_bias,
                      a->d_bias,
                      a->table,
                      a->q_norm_weight,
                      a->k_norm_weight,
                      a->hk_in,
                      a->hv_in,
                      a->clock_in,
                      a->hk_out,
                      a->hv_out,
                      a->clock_out,
                      static_cast<const __nv_bfloat16*>(a->gate),
                      static_cast<const __nv_bfloat16*>(a->gate_bias),
                      a->o_norm_weight,
                      static_cast<__nv_bfloat16*>(a->y),
                      B,
                      H,
                      a->q_eps,
                      a->k_eps,
                      a->scale,
                      a->o_eps,
                      a->o_scale};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid(B * H);
#define CYFA_DL(KK, VV, WW) \
  CYFA_LAUNCH("decode_layer", s, (launch_k(decode_layer_kernel<KK, VV, WW>, grid, 256, 0, s, p)))
#define CYFA_DL_W(KK, VV) \
  if (W == 2) CYFA_DL(KK, VV, 2); else if (W == 3) CYFA_DL(KK, VV, 3); else CYFA_DL(KK, VV, 4)
  if (K == 256 && V == 256) { CYFA_DL_W(256, 256); }
  else if (K == 128 && V == 128) { CYFA_DL_W(128, 128); }
  else if (K == 256) { CYFA_DL_W(256, 128); }
  else { CYFA_DL_W(128, 256); }
#undef CYFA_DL_W
#undef CYFA_DL
  return launch_status();
}

int cyfa_add_rmsnorm(void* x, const void* y, const float* w, float eps, void* out, int rows,
                     int D, void* stream) {
  CYFA_REQUIRE(x && w && out, kNullPointer);
  CYFA_REQUIRE(rows > 0 && D > 0 && D % 8 == 0 && D <= 8192, kBadShape);
  CYFA_REQUIRE(aligned(x, 16) && aligned(out, 16) && aligned(w, 16) && (!y || aligned(y, 16)),
               kMisaligned);
  AddNormParams p{static_cast<__nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(y), w,
                  static_cast<__nv_bfloat16*>(out), eps, rows, D};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CYFA_LAUNCH("add_rmsnorm", s,
              (launch_k(add_rmsnorm_kernel, unsigned(rows), 256, 0, s, p)));
  return launch_status();
}

int cyfa_decode_conv(const void* x, long long x_stride, void* cache_q, void* cache_k,
                     void* cache_v, const float* wq, const float* wk, const float* wv, void* yq,
                     void* yk, void* yv, int B, int Cq, int Ck, int Cv, int W, void* stream) {
  CYFA_REQUIRE(x && cache_q && cache_k && cache_v && wq && wk && wv && yq && yk && yv,
               kNullPointer);
  CYFA_REQUIRE(B > 0 && W >= 2 && W <= 4 && Cq > 0 && Ck > 0 && Cv > 0 && Cq % 8 == 0 &&
                   Ck % 8 == 0 && Cv % 8 == 0 && x_stride >= (long long)Cq + Ck + Cv &&
                   x_stride % 8 == 0,
               kBadShape);
  CYFA_REQUIRE(aligned(x, 16) && aligned(cache_q, 16) && aligned(cache_k, 16) &&
                   aligned(cache_v, 16) && aligned(yq, 16) && aligned(yk, 16) && aligned(yv, 16) &&
                   aligned(wq, 16) && aligned(wk, 16) && aligned(wv, 16),
               kMisaligned);
  DecodeConvParams p{static_cast<const __nv_bfloat16*>(x),
                     x_stride,
                     {static_cast<__nv_bfloat16*>(cache_q), static_cast<__nv_bfloat16*>(cache_k),
                      static_cast<__nv_bfloat16*>(cache_v)},
                     {wq, wk, wv},
                     {static_cast<__nv_bfloat16*>(yq), static_cast<__nv_bfloat16*>(yk),
                      static_cast<__nv_bfloat16*>(yv)},
                     {Cq, Ck, Cv},
                     B,
                     W};
  const long long n = (long long)B * ((Cq + Ck + Cv) / 8);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned grid = unsigned((n + 255) / 256);
  if (W == 2) CYFA_LAUNCH("decode_conv", s, (launch_k(decode_conv_kernel<2>, grid, 256, 0, s, p)));
  else if (W == 3) CYFA_LAUNCH("decode_conv", s, (launch_k(decode_conv_kernel<3>, grid, 256, 0, s, p)));
  else CYFA_LAUNCH("decode_conv", s, (launch_k(decode_conv_kernel<4>, grid, 256, 0, s, p)));
  return launch_status();
}

int cyfa_swiglu(const void* gu, void* out, int rows, int mid, void* stream) {
  CYFA_REQUIRE(gu && out, kNullPointer);
  CYFA_REQUIRE(rows > 0 && mid > 0 && mid % 8 == 0, kBadShape);
  CYFA_REQUIRE(aligned(gu, 16) && aligned(out, 16), kMisaligned);
  SwigluParams p{static_cast<const __nv_bfloat16*>(gu), static_cast<__nv_bfloat16*>(out), rows,
                 mid};
  const long long n = (long long)rows * (mid / 8);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CYFA_LAUNCH("swiglu", s, (launch_k(swiglu_kernel, unsigned((n + 255) / 256), 256, 0, s, p)));
  return launch_status();
}

}  // extern "C"
