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

int cyfa_bucket_gather(const cyfa_bucket_piece* pieces, int count, float* flat, void* stream) {
  return bucket_launch(pieces, count, flat, 1.f, true, static_cast<cudaStream_t>(stream));
}

int cyfa_bucket_scatter(const cyfa_bucket_piece* pieces, int count, const float* flat,
                        float scale, void* stream) {
  return bucket_launch(pieces, count, const_cast<float*>(flat), scale, false,
                       static_cast<cudaStream_t>(stream));
}

}  // extern "C"
