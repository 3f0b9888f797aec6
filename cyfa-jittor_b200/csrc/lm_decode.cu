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

extern "C" {

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
