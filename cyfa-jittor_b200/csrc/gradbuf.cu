// Gradient buckets for data-parallel training: one launch gathers the
// gradients of up to kMaxPieces tensors (bf16 or f32) into a flat fp32 bucket
// for the all-reduce, and one launch scatters the averaged bucket back,
// converting to each tensor's dtype.  The reference flattens its fp32 bucket
// with framework ops (training/optim.py:52-63); here the copies are one kernel
// per bucket instead of one per tensor.
#include "cyfa_common.cuh"

namespace cyfa {

constexpr int kMaxPieces = 64;
constexpr int kBucketChunk = 2048;  // elements per block: 256 threads x 8

struct BucketArgs {
  int count;
  int blk_prefix[kMaxPieces + 1];  // first block of each piece
  void* ptr[kMaxPieces];
  long long n[kMaxPieces];
  long long off[kMaxPieces];
  int dtype[kMaxPieces];  // 0 = f32, 1 = bf16
  float* flat;
  float scale;
};

__device__ __forceinline__ int bucket_piece(const BucketArgs& a, int b) {
  int lo = 0, hi = a.count - 1;
  while (lo < hi) {  // last piece whose first block is <= b
    const int mid = (lo + hi + 1) >> 1;
    if (a.blk_prefix[mid] <= b) lo = mid; else hi = mid - 1;
  }
  return lo;
}

template <bool GATHER>
__global__ void __launch_bounds__(256) bucket_copy_kernel(const __grid_constant__ BucketArgs a) {
  pdl_wait();
  pdl_trigger();
  const int i = bucket_piece(a, blockIdx.x);
  const long long e0 = (long long)(blockIdx.x - a.blk_prefix[i]) * kBucketChunk + threadIdx.x * 8;
  const long long n = a.n[i];
  if (e0 >= n) return;
  float* flat = a.flat + a.off[i] + e0;
  const bool bf = a.dtype[i] == 1;
  if (e0 + 8 <= n) {
    if (GATHER) {
      float v[8];
      if (bf) {
        unpack_bf16x8(*reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.ptr[i]) + e0), v);
      } else {
        const float4* s = reinterpret_cast<const float4*>(static_cast<const float*>(a.ptr[i]) + e0);
        const float4 x = s[0], y = s[1];
        v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w; v[4] = y.x; v[5] = y.y; v[6] = y.z; v[7] = y.w;
      }
      float4* d = reinterpret_cast<float4*>(flat);
      d[0] = make_float4(v[0], v[1], v[2], v[3]);
      d[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
      const float4* s = reinterpret_cast<const float4*>(flat);
      const float4 x = s[0], y = s[1];
      float v[8] = {x.x, x.y, x.z, x.w, y.x, y.y, y.z, y.w};
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] *= a.scale;
      if (bf) {
        uint4 o;
        uint32_t* w = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
          w[k] = *reinterpret_cast<uint32_t*>(&h);
        }
        *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.ptr[i]) + e0) = o;
      } else {
        float4* d = reinterpret_cast<float4*>(static_cast<float*>(a.ptr[i]) + e0);
        d[0] = make_float4(v[0], v[1], v[2], v[3]);
        d[1] = make_float4(v[4], v[5], v[6], v[7]);
      }
    }
    return;
  }
  for (long long e = e0; e < n; ++e) {  // ragged tail of a piece
    const long long k = e - e0;
    if (GATHER) {
      flat[k] = bf ? __bfloat162float(static_cast<const __nv_bfloat16*>(a.ptr[i])[e])
                   : static_cast<const float*>(a.ptr[i])[e];
    } else {
      const float v = flat[k] * a.scale;
      if (bf) static_cast<__nv_bfloat16*>(a.ptr[i])[e] = __float2bfloat16_rn(v);
      else static_cast<float*>(a.ptr[i])[e] = v;
    }
  }
}

// ---------------------------------------------------------------- AdamW
// One launch updates every parameter of a group: the fp32 master weights and
// moments live in flat buffers laid out like a gradient bucket (each parameter
// at its piece offset, a multiple of 8); the parameter itself receives the new
// master value rounded to its dtype.  Per element, in the reference's order
// (training/optim.py:96-121):
//   m = b0 m + (1 - b0) g;  v = b1 v + (1 - b1) g g
//   master = master (1 - lr decay) - (lr / bc1) m / (sqrt(v / bc2) + eps)
__device__ __forceinline__ void load8(const float* p, float* f) {
  const float4 x = reinterpret_cast<const float4*>(p)[0], y = reinterpret_cast<const float4*>(p)[1];
  f[0] = x.x; f[1] = x.y; f[2] = x.z; f[3] = x.w; f[4] = y.x; f[5] = y.y; f[6] = y.z; f[7] = y.w;
}
__device__ __forceinline__ void store8(float* p, const float* f) {
  reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
}

struct AdamArgs {
  BucketArgs pieces;  // ptr = the parameters, off = offsets into the flat buffers
  float* master;
  float* m;
  float* v;
  const float* grad;
  float b0, b1, eps, shrink, step_size, bc2;  // shrink = 1 - lr decay, step_size = lr / bc1
};

__device__ __forceinline__ void adam_one(float& w, float& m, float& v, float g, const AdamArgs& a) {
  m = a.b0 * m + (1.f - a.b0) * g;
  v = a.b1 * v + (1.f - a.b1) * g * g;
  w = w * a.shrink - a.step_size * m / (sqrtf(v / a.bc2) + a.eps);
}

__global__ void __launch_bounds__(256) adamw_kernel(const __grid_constant__ AdamArgs a) {
  pdl_wait();
  pdl_trigger();
  const BucketArgs& pc = a.pieces;
  const int i = bucket_piece(pc, blockIdx.x);
  const long long e0 = (long long)(blockIdx.x - pc.blk_prefix[i]) * kBucketChunk + threadIdx.x * 8;
  const long long n = pc.n[i];
  if (e0 >= n) return;
  const long long f = pc.off[i] + e0;
  const bool bf = pc.dtype[i] == 1;
  if (e0 + 8 <= n) {
    float w[8], m[8], v[8], g[8];
    load8(a.master + f, w);
    load8(a.m + f, m);
    load8(a.v + f, v);
    load8(a.grad + f, g);
#pragma unroll
    for (int k = 0; k < 8; ++k) adam_one(w[k], m[k], v[k], g[k], a);
    store8(a.master + f, w);
    store8(a.m + f, m);
    store8(a.v + f, v);
    if (bf) {
      uint4 o;
      uint32_t* u = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        __nv_bfloat162 h = __floats2bfloat162_rn(w[2 * k], w[2 * k + 1]);
        u[k] = *reinterpret_cast<uint32_t*>(&h);
      }
      *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(pc.ptr[i]) + e0) = o;
    } else {
      store8(static_cast<float*>(pc.ptr[i]) + e0, w);
    }
    return;
  }
  for (long long e = e0; e < n; ++e) {  // ragged tail of a piece
    const long long k = f + e - e0;
    float w = a.master[k], m = a.m[k], v = a.v[k];
    adam_one(w, m, v, a.grad[k], a);
    a.master[k] = w;
    a.m[k] = m;
    a.v[k] = v;
    if (bf) static_cast<__nv_bfloat16*>(pc.ptr[i])[e] = __float2bfloat16_rn(w);
    else static_cast<float*>(pc.ptr[i])[e] = w;
  }
}

// ---------------------------------------------------------------- gradient clipping
// L2 norm of a flat fp32 gradient buffer in a fixed order (per-block partial sums
// of squares, then one block sums them), the clip coefficient
// min(max_norm / (norm + 1e-6), 1) (training/optim.py:74-89), and the in-place
// scaling by it.
constexpr int kNormBlocks = 592;  // 4 x 148 SMs

__global__ void __launch_bounds__(256) sumsq_kernel(const float* x, long long n, float* part) {
  pdl_wait();
  pdl_trigger();
  float s = 0.f;
  for (long long i = (long long)blockIdx.x * 256 + threadIdx.x; i < n; i += (long long)gridDim.x * 256)
    s = fmaf(x[i], x[i], s);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  __shared__ float ws[8];
  if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += ws[w];
    part[blockIdx.x] = t;
  }
}

__global__ void __launch_bounds__(1024) clip_coef_kernel(const float* part, int nparts, float max_norm,
                                                        float* coef, float* norm_out) {
  pdl_wait();
  pdl_trigger();
  float s = 0.f;
  for (int i = threadIdx.x; i < nparts; i += 1024) s += part[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  __shared__ float ws[32];
  if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < 32; ++w) t += ws[w];
    const float norm = sqrtf(t);
    *coef = fminf(max_norm / (norm + 1e-6f), 1.f);
    if (norm_out) *norm_out = norm;
  }
}

__global__ void __launch_bounds__(256) scale_kernel(float* x, long long n, const float* coef) {
  pdl_wait();
  pdl_trigger();
  const float c = *coef;
  for (long long i = (long long)blockIdx.x * 256 + threadIdx.x; i < n; i += (long long)gridDim.x * 256)
    x[i] *= c;
}

}  // namespace cyfa

using namespace cyfa;

static int bucket_launch(const cyfa_bucket_piece* pieces, int count, float* flat, float scale,
                         bool gather, cudaStream_t st) {
  CYFA_REQUIRE(count >= 0, kBadShape);
  CYFA_REQUIRE(count == 0 || (pieces && flat), kNullPointer);
  CYFA_REQUIRE(aligned(flat, 16), kMisaligned);
  for (int base = 0; base < count; base += kMaxPieces) {
    BucketArgs a{};
    a.count = count - base < kMaxPieces ? count - base : kMaxPieces;
    a.flat = flat;
    a.scale = scale;
    long long blocks = 0;
    for (int i = 0; i < a.count; ++i) {
      const cyfa_bucket_piece& p = pieces[base + i];
      CYFA_REQUIRE(p.n >= 0 && p.offset >= 0, kBadShape);
      CYFA_REQUIRE(p.dtype == 0 || p.dtype == 1, kBadDtype);
      CYFA_REQUIRE(p.n == 0 || p.ptr, kNullPointer);
      CYFA_REQUIRE(aligned(p.ptr, 16) && p.offset % 8 == 0, kMisaligned);
      a.blk_prefix[i] = static_cast<int>(blocks);
      a.ptr[i] = p.ptr;
      a.n[i] = p.n;
      a.off[i] = p.offset;
      a.dtype[i] = p.dtype;
      blocks += (p.n + kBucketChunk - 1) / kBucketChunk;
      CYFA_REQUIRE(blocks < (1LL << 30), kBadShape);
    }
    a.blk_prefix[a.count] = static_cast<int>(blocks);
    if (blocks == 0) continue;
    if (gather) {
      CYFA_LAUNCH("bucket_gather", st, (launch_k(bucket_copy_kernel<true>, unsigned(blocks), 256, 0, st, a)));
    } else {
      CYFA_LAUNCH("bucket_scatter", st, (launch_k(bucket_copy_kernel<false>, unsigned(blocks), 256, 0, st, a)));
    }
    const int s = launch_status();
    if (s != kOk) return s;
  }
  return kOk;
}

extern "C" {

int cyfa_adamw_step(const cyfa_bucket_piece* params, int count, float* master, float* m, float* v,
                    const float* grad, float lr, float beta1, float beta2, float eps,
                    float weight_decay, int step, void* stream) {
  CYFA_REQUIRE(count >= 0 && step >= 1, kBadShape);
  CYFA_REQUIRE(count == 0 || (params && master && m && v && grad), kNullPointer);
  CYFA_REQUIRE(aligned(master, 16) && aligned(m, 16) && aligned(v, 16) && aligned(grad, 16),
               kMisaligned);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float bc1 = 1.f - powf(beta1, float(step));
  const float bc2 = 1.f - powf(beta2, float(step));
  for (int base = 0; base < count; base += kMaxPieces) {
    AdamArgs a{};
    BucketArgs& pc = a.pieces;
    pc.count = count - base < kMaxPieces ? count - base : kMaxPieces;
    long long blocks = 0;
    for (int i = 0; i < pc.count; ++i) {
      const cyfa_bucket_piece& p = params[base + i];
      CYFA_REQUIRE(p.n >= 0 && p.offset >= 0, kBadShape);
      CYFA_REQUIRE(p.dtype == 0 || p.dtype == 1, kBadDtype);
      CYFA_REQUIRE(p.n == 0 || p.ptr, kNullPointer);
      CYFA_REQUIRE(aligned(p.ptr, 16) && p.offset % 8 == 0, kMisaligned);
      pc.blk_prefix[i] = static_cast<int>(blocks);
      pc.ptr[i] = p.ptr;
      pc.n[i] = p.n;
      pc.off[i] = p.offset;
      pc.dtype[i] = p.dtype;
      blocks += (p.n + kBucketChunk - 1) / kBucketChunk;
      CYFA_REQUIRE(blocks < (1LL << 30), kBadShape);
    }
    pc.blk_prefix[pc.count] = static_cast<int>(blocks);
    if (blocks == 0) continue;
    a.master = master;
    a.m = m;
    a.v = v;
    a.grad = grad;
    a.b0 = beta1;
    a.b1 = beta2;
    a.eps = eps;
    a.shrink = 1.f - lr * weight_decay;
    a.step_size = lr / bc1;
    a.bc2 = bc2;
    CYFA_LAUNCH("adamw", st, (launch_k(adamw_kernel, unsigned(blocks), 256, 0, st, a)));
    const int rc = launch_status();
    if (rc != kOk) return rc;
  }
  return kOk;
}

size_t cyfa_grad_clip_work_bytes(void) { return (kNormBlocks + 4) * sizeof(float); }

int cyfa_grad_clip(float* grad, long long n, float max_norm, float* norm_out, void* work,
                   size_t work_bytes, void* stream) {
  CYFA_REQUIRE(n >= 0 && max_norm > 0.f, kBadShape);
  CYFA_REQUIRE(n == 0 || grad, kNullPointer);
  CYFA_REQUIRE(work && work_bytes >= cyfa_grad_clip_work_bytes(), kWorkspace);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float* part = static_cast<float*>(work);
  float* coef = part + kNormBlocks;
  CYFA_LAUNCH("grad_sumsq", st, (launch_k(sumsq_kernel, kNormBlocks, 256, 0, st,
                                          static_cast<const float*>(grad), n, part)));
  int rc = launch_status();
  if (rc) return rc;
  CYFA_LAUNCH("grad_clip_coef", st, (launch_k(clip_coef_kernel, 1, 1024, 0, st,
                                              static_cast<const float*>(part), kNormBlocks,
                                              max_norm, coef, norm_out)));
  rc = launch_status();
  if (rc) return rc;
  CYFA_LAUNCH("grad_scale", st, (launch_k(scale_kernel, kNormBlocks, 256, 0, st, grad, n,
                                          static_cast<const float*>(coef))));
  return launch_status();
}

int cyfa_bucket_gather(const cyfa_bucket_piece* pieces, int count, float* flat, void* stream) {
  return bucket_launch(pieces, count, flat, 1.f, true, static_cast<cudaStream_t>(stream));
}

int cyfa_bucket_scatter(const cyfa_bucket_piece* pieces, int count, const float* flat,
                        float scale, void* stream) {
  return bucket_launch(pieces, count, const_cast<float*>(flat), scale, false,
                       static_cast<cudaStream_t>(stream));
}

}  // extern "C"
