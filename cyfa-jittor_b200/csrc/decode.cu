// Constant-memory CyFA decode step (T = 1), replacing the reference's fused
// decode kernel (cyclic_flow_attention/ops/fused_recurrent.py:55-188).
//
// One CTA of 256 threads per (batch, head).  The step is HBM-bound: it reads and
// writes the fp32 key state hk [K, 128] and value state hv [128, V] once each
// (512 KiB per (b,h) at K = V = 256).  Both sweeps use 16-byte vector loads that
// are coalesced along the contiguous dimension and unrolled for memory-level
// parallelism:
//   sweep 1: hk' = a hk + k^ w^T and raw = scale hk'^T q^   (threads over m-quads x d-groups)
//   readout: z = U(lam) raw, logits = Table z, softmax over 127, coeff = p Table,
//            weights = U(-lam) coeff                        (warp-cooperative dots)
//   sweep 2: hv' = a hv + w v^T and o = hv'^T weights        (threads over v-quads x m-groups)
// The rounding points follow the reference decode: normalised q/k, the write
// vector, the rotated raw vector, the probabilities, the table and the weights
// are rounded to the input dtype; states and accumulations stay fp32.
#include "cyfa_common.cuh"
#include "phase.cuh"

namespace cyfa {

struct DecodeParams {
  const void* q;      // [B*H, K]  (input layout [B,1,H,K])
  const void* k;      // [B*H, K]
  const void* v;      // [B*H, V]
  const float* g;     // [B*H] log decay
  const float* delta; // [B*H]
  const float* beta;  // [B*H]
  const float* table; // [H, 127, 128] fp32 readout table R.Phi
  const float* q_norm_weight;  // [K]
  const float* k_norm_weight;  // [K]
  const float* hk_in;  // [B*H, K, 128] or null (zero state)
  const float* hv_in;  // [B*H, 128, V] or null
  const float* clock_in;  // [B*H] or null
  float* hk_out;
  float* hv_out;
  float* clock_out;
  void* out;  // [B*H, V]
  int BH, H;
  float q_eps, k_eps, scale;
};

template <typename T>
__device__ __forceinline__ float to_f(T x);
template <>
__device__ __forceinline__ float to_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

// Rounds to the input dtype (identity for fp32 inputs).
template <typename T>
__device__ __forceinline__ float round_in(float x);
template <>
__device__ __forceinline__ float round_in<float>(float x) { return x; }
template <>
__device__ __forceinline__ float round_in<__nv_bfloat16>(float x) { return bf16_round(x); }

template <typename T>
__device__ __forceinline__ void store_out(void* p, int i, float x);
template <>
__device__ __forceinline__ void store_out<float>(void* p, int i, float x) { static_cast<float*>(p)[i] = x; }
template <>
__device__ __forceinline__ void store_out<__nv_bfloat16>(void* p, int i, float x) {
  static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(x);
}

__device__ __forceinline__ float block_sum_256(float x, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = x;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) s += red[i];
  return s;
}

__device__ __forceinline__ float block_max_256(float x, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = x;
  __syncthreads();
  float s = red[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) s = fmaxf(s, red[i]);
  return s;
}

// One token of one (batch, head): the whole decode step on this CTA's 256
// threads.  Each thread reads and writes the same state elements in both sweeps,
// so the state may be updated in place (src == dst) with no barrier; the shared
// scratch is reused by the next call only after its trailing barrier.
struct TokenIO {
  const void* q;        // this token's q row [K]
  const void* k;        // [K]
  const void* v;        // [V]
  float g, beta, lam;   // log decay, write strength, clock after this token
  const float* hk_src;  // [K, 128] or null (zero state)
  const float* hv_src;  // [128, V] or null
  float* hk_dst;
  float* hv_dst;
  float* clock_dst;     // stores lam once every thread has read the clock, or null
  void* out;            // output row [V]
};

// kStream: streaming cache hints for states touched once (decode); the chunk
// loop keeps its per-(b,h) state resident in L2 instead.
template <typename Tin, int K, int V, bool kStream>
__device__ __forceinline__ void decode_token(const TokenIO& io, const float* tab,
                                             const float* qnw, const float* knw, float q_eps,
                                             float k_eps, float scale) {
  constexpr int M = 128;
  const int tid = threadIdx.x;
  __shared__ float sq[K], sk[K];
  // per-group partial sums (sweep 1 uses 8x128, sweep 2 4x256), written as float4:
  // 16-byte alignment is required whatever other shared arrays the kernel declares
  __shared__ __align__(16) float part[8 * M];
  __shared__ float wv[M], raw[M], z[M], wts[M], prob[128];
  __shared__ float red[8];

  const Tin* q = static_cast<const Tin*>(io.q);
  const Tin* kk = static_cast<const Tin*>(io.k);
  const Tin* vv = static_cast<const Tin*>(io.v);

  // ---- q/k RMSNorm (head_dim K), rounded to the input dtype (ref :63-89)
  float q2 = 0.f, k2 = 0.f;
  for (int d = tid; d < K; d += 256) {
    const float a = to_f(q[d]), b = to_f(kk[d]);
    q2 += a * a;
    k2 += b * b;
  }
  const float qs = block_sum_256(q2, red);
  const float ks = block_sum_256(k2, red);
  const float qr = rsqrtf(qs / K + q_eps), kr = rsqrtf(ks / K + k_eps);
  for (int d = tid; d < K; d += 256) {
    sq[d] = round_in<Tin>(to_f(q[d]) * qr * qnw[d]) * scale;
    sk[d] = round_in<Tin>(to_f(kk[d]) * kr * knw[d]);
  }
  const float lam = io.lam;
  const float alpha = expf(io.g);
  const float bt = io.beta;
  if (tid < M) {
    const int pair = tid >> 1;
    float s, c;
    sincosf(clock_phase(lam, pair), &s, &c);
    wv[tid] = round_in<Tin>(bt * atom_scale(pair) * ((tid & 1) ? -s : c));
  }
  __syncthreads();
  // the clock output may alias the clock input (in-place decode): store only
  // after the barrier above, by which every thread has read the clock input
  if (tid == 0 && io.clock_dst) *io.clock_dst = lam;

  // ---- sweep 1: hk' = a hk + k^ w^T ; raw = hk'^T q^   (ref :94-112)
  {
    const int mq = tid & 31, dg = tid >> 5;  // 4 m values, 8 d-groups
    const float4 w4 = make_float4(wv[4 * mq], wv[4 * mq + 1], wv[4 * mq + 2], wv[4 * mq + 3]);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    const float4* src = reinterpret_cast<const float4*>(io.hk_src);
    float4* dst = reinterpret_cast<float4*>(io.hk_dst);
    constexpr int ROWS = K / 8;
    constexpr int U = 8;
#pragma unroll 1
    for (int i0 = 0; i0 < ROWS; i0 += U) {
      float4 x[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int d = dg + 8 * (i0 + u);
        x[u] = src ? (kStream ? __ldcs(src + d * (M / 4) + mq) : __ldcg(src + d * (M / 4) + mq))
                   : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int d = dg + 8 * (i0 + u);
        const float kd = sk[d], qd = sq[d];
        float4 y;
        y.x = x[u].x * alpha + kd * w4.x;
        y.y = x[u].y * alpha + kd * w4.y;
        y.z = x[u].z * alpha + kd * w4.z;
        y.w = x[u].w * alpha + kd * w4.w;
        if (kStream) __stcs(dst + d * (M / 4) + mq, y);
        else __stcg(dst + d * (M / 4) + mq, y);
        acc.x += y.x * qd;
        acc.y += y.y * qd;
        acc.z += y.z * qd;
        acc.w += y.w * qd;
      }
    }
    reinterpret_cast<float4*>(part)[dg * (M / 4) + mq] = acc;
  }
  __syncthreads();
  if (tid < M) {
    float s = 0.f;
#pragma unroll
    for (int gidx = 0; gidx < 8; ++gidx) s += part[gidx * M + tid];
    raw[tid] = s;
  }
  __syncthreads();

  // ---- readout (ref :114-175)
  if (tid < M) {
    const int pair = tid >> 1;
    float s, c;
    sincosf(clock_phase(lam, pair), &s, &c);
    const float e = raw[tid & ~1], o = raw[tid | 1];
    z[tid] = round_in<Tin>((tid & 1) ? s * e + c * o : c * e - s * o);
  }
  __syncthreads();
  {
    const int w = tid >> 5, l = tid & 31;
    for (int r = w; r < 127; r += 8) {
      const float4 t4 = reinterpret_cast<const float4*>(tab + r * M)[l];
      float s = round_in<Tin>(t4.x) * z[4 * l] + round_in<Tin>(t4.y) * z[4 * l + 1] +
                round_in<Tin>(t4.z) * z[4 * l + 2] + round_in<Tin>(t4.w) * z[4 * l + 3];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (l == 0) prob[r] = s;
    }
  }
  __syncthreads();
  const float logit = tid < 127 ? prob[tid] : -1e30f;
  const float mx = block_max_256(logit, red);
  const float e = tid < 127 ? expf(logit - mx) : 0.f;
  const float den = block_sum_256(e, red);
  if (tid < 128) prob[tid] = round_in<Tin>(e / den);
  __syncthreads();
  if (tid < M) {
    float s = 0.f;
    for (int r = 0; r < 127; ++r) s += prob[r] * round_in<Tin>(tab[r * M + tid]);
    raw[tid] = s;  // coeff
  }
  __syncthreads();
  if (tid < M) {
    const int pair = tid >> 1;
    float s, c;
    sincosf(clock_phase(lam, pair), &s, &c);
    const float e2 = raw[tid & ~1], o2 = raw[tid | 1];
    wts[tid] = round_in<Tin>((tid & 1) ? -s * e2 + c * o2 : c * e2 + s * o2);
  }
  __syncthreads();

  // ---- sweep 2: hv' = a hv + w v^T ; o = hv'^T weights  (ref :177-186)
  {
    constexpr int VQ = V / 4;         // float4 columns per row
    constexpr int MG = 256 / VQ;      // m-groups
    const int vq = tid % VQ, mg = tid / VQ;
    const float4 v4 = make_float4(to_f(vv[4 * vq]), to_f(vv[4 * vq + 1]), to_f(vv[4 * vq + 2]),
                                  to_f(vv[4 * vq + 3]));
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    const float4* src = reinterpret_cast<const float4*>(io.hv_src);
    float4* dst = reinterpret_cast<float4*>(io.hv_dst);
    constexpr int ROWS = M / MG;
    constexpr int U = 8;
#pragma unroll 1
    for (int i0 = 0; i0 < ROWS; i0 += U) {
      float4 x[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int m = mg + MG * (i0 + u);
        x[u] = src ? (kStream ? __ldcs(src + m * VQ + vq) : __ldcg(src + m * VQ + vq))
                   : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int m = mg + MG * (i0 + u);
        const float wm = wv[m], am = wts[m];
        float4 y;
        y.x = x[u].x * alpha + wm * v4.x;
        y.y = x[u].y * alpha + wm * v4.y;
        y.z = x[u].z * alpha + wm * v4.z;
        y.w = x[u].w * alpha + wm * v4.w;
        if (kStream) __stcs(dst + m * VQ + vq, y);
        else __stcg(dst + m * VQ + vq, y);
        acc.x += am * y.x;
        acc.y += am * y.y;
        acc.z += am * y.z;
        acc.w += am * y.w;
      }
    }
    __syncthreads();
    reinterpret_cast<float4*>(part)[mg * VQ + vq] = acc;
    __syncthreads();
    if (tid < V) {
      float s = 0.f;
#pragma unroll
      for (int gidx = 0; gidx < MG; ++gidx) s += part[gidx * V + tid];
      store_out<Tin>(io.out, tid, s);
    }
  }
  __syncthreads();  // the next token may overwrite the shared scratch
}

template <typename Tin, int K, int V>
__global__ void __launch_bounds__(256) decode_step_kernel(DecodeParams p) {
  pdl_wait();
  pdl_trigger();
  constexpr int M = 128;
  const int bh = blockIdx.x;
  const int h = bh % p.H;
  TokenIO io;
  io.q = static_cast<const Tin*>(p.q) + size_t(bh) * K;
  io.k = static_cast<const Tin*>(p.k) + size_t(bh) * K;
  io.v = static_cast<const Tin*>(p.v) + size_t(bh) * V;
  io.g = p.g[bh];
  io.beta = p.beta[bh];
  io.lam = (p.clock_in ? p.clock_in[bh] : 0.f) + p.delta[bh];
  io.hk_src = p.hk_in ? p.hk_in + size_t(bh) * K * M : nullptr;
  io.hv_src = p.hv_in ? p.hv_in + size_t(bh) * M * V : nullptr;
  io.hk_dst = p.hk_out + size_t(bh) * K * M;
  io.hv_dst = p.hv_out + size_t(bh) * M * V;
  io.clock_dst = p.clock_out + bh;
  io.out = static_cast<Tin*>(p.out) + size_t(bh) * V;
  decode_token<Tin, K, V, true>(io, p.table + size_t(h) * 127 * M, p.q_norm_weight,
                                p.k_norm_weight, p.q_eps, p.k_eps, p.scale);
}

// fp32 chunk forward as the token recurrence: one CTA of 256 threads per
// (batch, head) runs the decode step over all T tokens of its sequence, keeping
// its states in the caller's final-state buffers (512 KiB per (b, h) at
// K = V = 256, resident in L2 between tokens).  Every product and sum is fp32,
// so the result equals the reference's fp32 chunkwise path
// (cyclic_flow_attention/ops/chunk.py:136-161,300-331) up to summation order.
// The clock follows the reference's order: the running sum of delta from zero,
// plus the initial clock (ops/chunk.py:254-256).
struct RecurrentParams {
  const float* q;      // [B, T, H, K]
  const float* k;      // [B, T, H, K]
  const float* v;      // [B, T, H, V]
  const float* g;      // [B, T, H]
  const float* delta;  // [B, T, H]
  const float* beta;   // [B, T, H]
  const float* table;  // [H, 127, 128] fp32
  const float* q_norm_weight;
  const float* k_norm_weight;
  const float* hk0;    // [B*H, K, 128] or null
  const float* hv0;    // [B*H, 128, V] or null
  const float* clock0; // [B*H] or null
  float* hk;           // [B*H, K, 128] running and final state
  float* hv;           // [B*H, 128, V]
  float* clock;        // [B*H]
  float* o;            // [B, T, H, V]
  int B, T, H;
  float q_eps, k_eps, scale;
};

template <int K, int V>
__global__ void __launch_bounds__(256) recurrent_fwd_f32_kernel(RecurrentParams p) {
  pdl_wait();
  pdl_trigger();
  constexpr int M = 128;
  const int bh = blockIdx.x;
  const int b = bh / p.H, h = bh % p.H;
  const float* tab = p.table + size_t(h) * 127 * M;
  float* hk = p.hk + size_t(bh) * K * M;
  float* hv = p.hv + size_t(bh) * M * V;
  const float c0 = p.clock0 ? p.clock0[bh] : 0.f;
  float csum = 0.f;
  for (int t = 0; t < p.T; ++t) {
    const size_t row = (size_t(b) * p.T + t) * p.H + h;
    TokenIO io;
    io.q = p.q + row * K;
    io.k = p.k + row * K;
    io.v = p.v + row * V;
    io.g = p.g[row];
    io.beta = p.beta[row];
    csum = __fadd_rn(csum, p.delta[row]);
    io.lam = __fadd_rn(csum, c0);
    io.hk_src = t ? hk : (p.hk0 ? p.hk0 + size_t(bh) * K * M : nullptr);
    io.hv_src = t ? hv : (p.hv0 ? p.hv0 + size_t(bh) * M * V : nullptr);
    io.hk_dst = hk;
    io.hv_dst = hv;
    io.clock_dst = nullptr;
    io.out = p.o + row * V;
    decode_token<float, K, V, false>(io, tab, p.q_norm_weight, p.k_norm_weight, p.q_eps,
                                     p.k_eps, p.scale);
  }
  if (threadIdx.x == 0) p.clock[bh] = __fadd_rn(csum, c0);
  if (p.T == 0) {
    // no tokens: the final state is the initial state
    const int n = K * M;
    for (int i = threadIdx.x; i < n; i += 256) hk[i] = p.hk0 ? p.hk0[size_t(bh) * n + i] : 0.f;
    for (int i = threadIdx.x; i < M * V; i += 256)
      hv[i] = p.hv0 ? p.hv0[size_t(bh) * M * V + i] : 0.f;
  }
}

template __global__ void recurrent_fwd_f32_kernel<256, 256>(RecurrentParams);
template __global__ void recurrent_fwd_f32_kernel<128, 128>(RecurrentParams);
template __global__ void recurrent_fwd_f32_kernel<256, 128>(RecurrentParams);
template __global__ void recurrent_fwd_f32_kernel<128, 256>(RecurrentParams);

template __global__ void decode_step_kernel<__nv_bfloat16, 256, 256>(DecodeParams);
template __global__ void decode_step_kernel<__nv_bfloat16, 128, 128>(DecodeParams);
template __global__ void decode_step_kernel<__nv_bfloat16, 256, 128>(DecodeParams);
template __global__ void decode_step_kernel<__nv_bfloat16, 128, 256>(DecodeParams);
template __global__ void decode_step_kernel<float, 256, 256>(DecodeParams);
template __global__ void decode_step_kernel<float, 128, 128>(DecodeParams);
template __global__ void decode_step_kernel<float, 256, 128>(DecodeParams);
template __global__ void decode_step_kernel<float, 128, 256>(DecodeParams);

}  // namespace cyfa
