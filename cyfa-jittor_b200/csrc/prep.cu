// Per-token preparation kernels of the chunked CyFA forward and their adjoints.
//
//  gates_fwd   : one CTA per (b,h).  Moves g/delta/beta from the public [B,T,H]
//                layout to head-major [B,H,TP] (zero padded), and computes with
//                fixed-order (deterministic) block scans
//                  lam_t = clock0 + sum_{s<=t} delta_s              (ops/utils.py:229-302)
//                  G_t   = log2(e) * sum_{s<=t, same 128-token tile} g_s   (ops/utils.py:495-520,
//                          with the chunk widened from 64 to 128 tokens)
//                  clock_T = clock0 + sum_t delta_t                  (ops/utils.py:305-348)
//  token_fwd   : one warp per (b,t,h).  Per-head RMSNorm of q and k into head-major
//                bf16 (ops/qk_norm.py:64-107) and the write vector
//                w_t = beta_t U(-lam_t) b (ops/utils.py:543-587) as bf16.
//  token_bwd   : adjoints of token_fwd: dq, dk (public layout), per-block partial
//                sums of the norm-weight gradients, and dlam, dbeta of the write
//                vector (ops/qk_norm.py:109-165, ops/utils.py:589-640).
//  gates_bwd   : one CTA per (b,h): ddelta = reverse cumsum of dlam (+ d clock_T),
//                dg = in-tile reverse cumsum of dG (dG taken w.r.t. the natural-log
//                in-tile gate cumsum, tile-end terms added), layout back to [B,T,H].
#include "cyfa_common.cuh"
#include "phase.cuh"

namespace cyfa {

constexpr float kLog2e = 1.4426950408889634f;

// Vector loads/stores of E = 4 or 8 consecutive elements (16/32-byte aligned rows).
template <int E>
__device__ __forceinline__ void load_bf16_vec(const __nv_bfloat16* p, float* f) {
  if constexpr (E == 8) {
    unpack_bf16x8(*reinterpret_cast<const uint4*>(p), f);
  } else {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
    f[0] = a.x;
    f[1] = a.y;
    f[2] = b.x;
    f[3] = b.y;
  }
}
template <int E>
__device__ __forceinline__ void load_f32_vec(const float* p, float* f) {
  const float4* q = reinterpret_cast<const float4*>(p);
#pragma unroll
  for (int i = 0; i < E / 4; ++i) {
    const float4 x = q[i];
    f[4 * i] = x.x;
    f[4 * i + 1] = x.y;
    f[4 * i + 2] = x.z;
    f[4 * i + 3] = x.w;
  }
}
template <int E>
__device__ __forceinline__ void store_bf16_vec(__nv_bfloat16* p, const float* f) {
  if constexpr (E == 8) {
    *reinterpret_cast<uint4*>(p) = make_uint4(pack_bf16(f[0], f[1]), pack_bf16(f[2], f[3]),
                                              pack_bf16(f[4], f[5]), pack_bf16(f[6], f[7]));
  } else {
    *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf16(f[0], f[1]), pack_bf16(f[2], f[3]));
  }
}

struct GatesParams {
  const float* g;       // [B,T,H]
  const float* delta;   // [B,T,H]
  const float* beta;    // [B,T,H]
  const float* clock0;  // [B,H] or null
  float* G;             // [B,H,TP] log2 in-tile cumsum
  float* lam;           // [B,H,TP]
  float* beta_h;        // [B,H,TP]
  float* clock_out;     // [B,H] or null
  int B, T, H, TP;
  const int* lengths;   // [B] valid tokens of each sequence (right padding), or null
};

// Block-wide scans of the gate kernels: 1024 threads = 32 warps cover 1024 tokens,
// i.e. 8 tiles of 128 tokens (4 warps each).  All sums run in a fixed order.
struct ScanPair {
  float tile;   // scan within the 128-token tile
  float block;  // scan within the 1024-token block
};

// Inclusive (REVERSE: suffix) scans of x; also returns the block total.
template <bool REVERSE>
__device__ __forceinline__ ScanPair scan1024(float x, float* wsum, float* total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = REVERSE ? __shfl_down_sync(0xffffffffu, x, o) : __shfl_up_sync(0xffffffffu, x, o);
    if (REVERSE ? (lane + o < 32) : (lane >= o)) x = __fadd_rn(x, y);
  }
  if (lane == (REVERSE ? 0 : 31)) wsum[w] = x;
  __syncthreads();
  // every warp scans the 32 warp sums with shuffles (a fixed tree order): the
  // block scan over all warps and the scan within each group of 4 warps (tile)
  const float ws = wsum[lane];
  float bs = ws, ts = ws;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = REVERSE ? __shfl_down_sync(0xffffffffu, bs, o) : __shfl_up_sync(0xffffffffu, bs, o);
    if (REVERSE ? (lane + o < 32) : (lane >= o)) bs = __fadd_rn(bs, y);
  }
#pragma unroll
  for (int o = 1; o < 4; o <<= 1) {
    const float y = REVERSE ? __shfl_down_sync(0xffffffffu, ts, o) : __shfl_up_sync(0xffffffffu, ts, o);
    if (REVERSE ? ((lane & 3) + o < 4) : ((lane & 3) >= o)) ts = __fadd_rn(ts, y);
  }
  // carries of warp w: the (tile / block) scans up to warp w - 1 (REVERSE: from w + 1)
  const int src = REVERSE ? w + 1 : w - 1;
  const bool first_b = REVERSE ? w == 31 : w == 0;
  const bool first_t = REVERSE ? (w & 3) == 3 : (w & 3) == 0;
  const float bsrc = __shfl_sync(0xffffffffu, bs, src & 31);
  const float tsrc = __shfl_sync(0xffffffffu, ts, src & 31);
  const float block_carry = first_b ? 0.f : bsrc;
  const float tile_carry = first_t ? 0.f : tsrc;
  const float tot = __shfl_sync(0xffffffffu, bs, REVERSE ? 0 : 31);
  __syncthreads();
  *total = tot;
  return {__fadd_rn(x, tile_carry), __fadd_rn(x, block_carry)};
}

// Grid (B*H, ceil(TP/1024)): CTA (bh, k) scans token block k.  The clock carry
// into the block (clock0 plus every earlier block's deltas) is summed by the CTA
// itself, thread i over column i of the earlier blocks, so the blocks of a
// sequence run side by side.
__global__ void __launch_bounds__(1024) gates_fwd_kernel(GatesParams p) {
  pdl_wait();
  pdl_trigger();
  const int bh = blockIdx.x, b = bh / p.H, h = bh % p.H, k = blockIdx.y;
  __shared__ float wsum[32];
  const size_t obase = size_t(bh) * p.TP;
  const int t = k * 1024 + threadIdx.x;
  // tokens past a sequence's length are neutral, like the padding up to TP
  const int Tb = p.lengths ? min(max(p.lengths[b], 0), p.T) : p.T;
  auto delta_at = [&](int tt) {
    return tt < Tb ? p.delta[(size_t(b) * p.T + tt) * p.H + h] : 0.f;
  };
  float gv = 0.f, dv = 0.f, bv = 0.f;
  if (t < Tb) {
    const size_t i = (size_t(b) * p.T + t) * p.H + h;
    gv = p.g[i];
    dv = p.delta[i];
    bv = p.beta[i];
  }
  float e[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  int kk = 0;
  for (; kk + 8 <= k; kk += 8)
#pragma unroll
    for (int u = 0; u < 8; ++u) e[u] += delta_at((kk + u) * 1024 + threadIdx.x);
  for (; kk < k; ++kk) e[0] += delta_at(kk * 1024 + threadIdx.x);
  const float earlier = ((e[0] + e[1]) + (e[2] + e[3])) + ((e[4] + e[5]) + (e[6] + e[7]));
  float tot, etot;
  const ScanPair gs = scan1024<false>(gv, wsum, &tot);
  const ScanPair ds = scan1024<false>(dv, wsum, &tot);
  scan1024<false>(earlier, wsum, &etot);
  const float clock = __fadd_rn(p.clock0 ? p.clock0[bh] : 0.f, etot);
  if (t < p.TP) {
    p.G[obase + t] = gs.tile * kLog2e;
    p.lam[obase + t] = __fadd_rn(clock, ds.block);
    p.beta_h[obase + t] = bv;
  }
  if (k == gridDim.y - 1 && threadIdx.x == 0 && p.clock_out) p.clock_out[bh] = __fadd_rn(clock, tot);
}

struct TokenFwdParams {
  const __nv_bfloat16* q;  // [B,T,H,K]
  const __nv_bfloat16* k;  // [B,T,H,K]
  const float* qw;         // [K]
  const float* kw;         // [K]
  const float* lam;        // [B,H,TP]
  const float* beta_h;     // [B,H,TP]
  __nv_bfloat16* qn;       // [B,H,TP,K]
  __nv_bfloat16* kn;       // [B,H,TP,K]
  __nv_bfloat16* w;        // [B,H,TP,128]
  float* q_rs;             // [B,H,TP]
  float* k_rs;             // [B,H,TP]
  int B, T, H, TP;
  float q_eps, k_eps;
  long long q_stride, k_stride;  // elements between consecutive tokens of q / k
};

// One warp per (b, h, t) row, grid-strided, two rows per iteration (all loads of
// both rows issued before any math); the norm weights stay in registers.
template <int K>
__global__ void __launch_bounds__(256) token_fwd_kernel(TokenFwdParams p) {
  pdl_wait();
  pdl_trigger();
  constexpr int E = K / 32;  // elements per lane (8 for K=256, 4 for K=128)
  const int lane = threadIdx.x & 31;
  const size_t rows = size_t(p.B) * p.H * p.TP;
  const size_t stride = size_t(gridDim.x) * 8;
  float qw[E], kw[E];
  load_f32_vec<E>(p.qw + lane * E, qw);
  load_f32_vec<E>(p.kw + lane * E, kw);
  for (size_t row0 = size_t(blockIdx.x) * 8 + (threadIdx.x >> 5); row0 < rows; row0 += 2 * stride) {
    float qv[2][E], kv[2][E], lam[2], bt[2];
    size_t rowv[2];
    bool live[2], real[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const size_t row = row0 + u * stride;
      rowv[u] = row;
      live[u] = row < rows;
      const int t = live[u] ? int(row % p.TP) : 0;
      real[u] = live[u] && t < p.T;
#pragma unroll
      for (int j = 0; j < E; ++j) qv[u][j] = kv[u][j] = 0.f;
      lam[u] = bt[u] = 0.f;
      if (real[u]) {
        const size_t bh = row / p.TP;
        const int b = int(bh / p.H), h = int(bh % p.H);
        const size_t tok = size_t(b) * p.T + t, col = size_t(h) * K + lane * E;
        load_bf16_vec<E>(p.q + tok * p.q_stride + col, qv[u]);
        load_bf16_vec<E>(p.k + tok * p.k_stride + col, kv[u]);
      }
      if (live[u]) {
        lam[u] = p.lam[row];
        bt[u] = p.beta_h[row];
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      if (!live[u]) continue;
      const size_t row = rowv[u];
      float q2 = 0.f, k2 = 0.f;
#pragma unroll
      for (int j = 0; j < E; ++j) {
        q2 += qv[u][j] * qv[u][j];
        k2 += kv[u][j] * kv[u][j];
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        q2 += __shfl_xor_sync(0xffffffffu, q2, o);
        k2 += __shfl_xor_sync(0xffffffffu, k2, o);
      }
      const float qr = rsqrtf(q2 / K + p.q_eps), kr = rsqrtf(k2 / K + p.k_eps);
      float qo[E], ko[E];
#pragma unroll
      for (int j = 0; j < E; ++j) {
        qo[j] = qv[u][j] * qr * qw[j];
        ko[j] = kv[u][j] * kr * kw[j];
      }
      store_bf16_vec<E>(p.qn + row * K + lane * E, qo);
      store_bf16_vec<E>(p.kn + row * K + lane * E, ko);
      if (lane == 0) {
        p.q_rs[row] = real[u] ? qr : 0.f;
        p.k_rs[row] = real[u] ? kr : 0.f;
      }
      // write vector: lane handles pairs lane and lane + 32 (|phase| <= pi)
      uint32_t wo[2];
#pragma unroll
      for (int part = 0; part < 2; ++part) {
        const int pair = lane + 32 * part;
        float sn, cs;
        __sincosf(clock_phase(lam[u], pair), &sn, &cs);
        const float a = bt[u] * atom_scale(pair);
        wo[part] = pack_bf16(a * cs, -a * sn);
      }
      uint32_t* wrow = reinterpret_cast<uint32_t*>(p.w + row * 128);
      wrow[lane] = wo[0];
      wrow[lane + 32] = wo[1];
    }
  }
}

// Blocks of token_fwd_kernel: enough for two rows per warp per pass, at most 8 per SM.
inline int token_fwd_blocks(size_t rows) {
  const size_t want = (rows + 15) / 16;
  return int(want < 1184 ? want : 1184);
}

template __global__ void token_fwd_kernel<256>(TokenFwdParams);
template __global__ void token_fwd_kernel<128>(TokenFwdParams);

// TMA-streamed token_fwd: persistent CTAs take 32-token tiles of one (b, h); warp
// 8 (one lane) loads the tile's q and k rows ([32, K] boxes of 3-D maps {H*K, T, B}
// over the token-strided inputs, rows past T read as zeros) into a shared ring,
// warps 0-7 take four tokens each with the norm weights in registers.  Same
// outputs and arithmetic as token_fwd_kernel.
constexpr int kTfRows = 32;
constexpr int kTfStages = 3;  // 97 KiB ring: two CTAs per SM

template <int K>
constexpr int token_fwd_tma_smem() {
  return kTfStages * 2 * kTfRows * K * 2 + 1024;
}

template <int K>
__global__ void __launch_bounds__(288, 2)
    token_fwd_tma_kernel(const __grid_constant__ CUtensorMap map_q,
                         const __grid_constant__ CUtensorMap map_k, TokenFwdParams p) {
  constexpr int E = K / 32;
  constexpr int kTile = kTfRows * K * 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[kTfStages], empty[kTfStages];
  __shared__ int s_abort;
  volatile int* abort_flag = &s_abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = p.TP / kTfRows, ntiles = p.B * p.H * nb;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kTfStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 8);
    }
    s_abort = 0;
    mbar_fence_init();
    prefetch_tmap(&map_q);
    prefetch_tmap(&map_k);
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();
  if (warp == 8) {
    if (lane == 0) {
      int issued = 0;
      for (int i = 0, k = blockIdx.x; k < ntiles; ++i, k += gridDim.x) {
        const int s = i % kTfStages;
        if (i >= kTfStages && !mbar_wait(&empty[s], ((i / kTfStages) - 1) & 1)) {
          *abort_flag = 1;
          break;
        }
        const int bh = k / nb, t0 = (k % nb) * kTfRows;
        uint8_t* st = smem + s * 2 * kTile;
        mbar_expect_tx(&full[s], 2 * kTile);
        tma_load_3d(st, &map_q, &full[s], (bh % p.H) * K, t0, bh / p.H);
        tma_load_3d(st + kTile, &map_k, &full[s], (bh % p.H) * K, t0, bh / p.H);
        issued = i + 1;
      }
      for (int i = issued > kTfStages ? issued - kTfStages : 0; i < issued; ++i)
        mbar_wait(&full[i % kTfStages], (i / kTfStages) & 1);
    }
    return;
  }
  float qw[E], kw[E];
  load_f32_vec<E>(p.qw + lane * E, qw);
  load_f32_vec<E>(p.kw + lane * E, kw);
  const int r0 = warp * 4;
  // lam and beta of the warp's four rows (lanes 0-3), one tile ahead
  auto scal = [&](int k) {
    float2 v = make_float2(0.f, 0.f);
    if (lane < 4 && k < ntiles) {
      const size_t row = size_t(k / nb) * p.TP + (k % nb) * kTfRows + r0 + lane;
      v = make_float2(p.lam[row], p.beta_h[row]);
    }
    return v;
  };
  float2 sc_cur = scal(blockIdx.x);
  for (int i = 0, k = blockIdx.x; k < ntiles; ++i, k += gridDim.x) {
    const float2 sc_next = scal(k + gridDim.x);
    const int s = i % kTfStages;
    const bool got = __all_sync(0xffffffffu, *abort_flag == 0 &&
                                                 mbar_wait(&full[s], (i / kTfStages) & 1));
    if (!got) {
      *abort_flag = 1;
      break;
    }
    const int bh = k / nb, t0 = (k % nb) * kTfRows;
    const uint8_t* st = smem + s * 2 * kTile;
    // the four rows' two norms reduced together
    float qv[4][E], kv[4][E], q2[4], k2[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int off = (r0 + u) * K * 2 + lane * E * 2;
      load_bf16_vec<E>(reinterpret_cast<const __nv_bfloat16*>(st + off), qv[u]);
      load_bf16_vec<E>(reinterpret_cast<const __nv_bfloat16*>(st + kTile + off), kv[u]);
      q2[u] = k2[u] = 0.f;
#pragma unroll
      for (int j = 0; j < E; ++j) {
        q2[u] += qv[u][j] * qv[u][j];
        k2[u] += kv[u][j] * kv[u][j];
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        q2[u] += __shfl_xor_sync(0xffffffffu, q2[u], o);
        k2[u] += __shfl_xor_sync(0xffffffffu, k2[u], o);
      }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int t = t0 + r0 + u;
      const bool real = t < p.T;
      const size_t row = size_t(bh) * p.TP + t;
      const float lam = __shfl_sync(0xffffffffu, sc_cur.x, u);
      const float bt = __shfl_sync(0xffffffffu, sc_cur.y, u);
      const float qr = rsqrtf(q2[u] / K + p.q_eps), kr = rsqrtf(k2[u] / K + p.k_eps);
      float qo[E], ko[E];
#pragma unroll
      for (int j = 0; j < E; ++j) {
        qo[j] = qv[u][j] * qr * qw[j];
        ko[j] = kv[u][j] * kr * kw[j];
      }
      store_bf16_vec<E>(p.qn + row * K + lane * E, qo);
      store_bf16_vec<E>(p.kn + row * K + lane * E, ko);
      if (lane == 0) {
        p.q_rs[row] = real ? qr : 0.f;
        p.k_rs[row] = real ? kr : 0.f;
      }
      // write vector: lane handles pairs lane and lane + 32 (|phase| <= pi)
      uint32_t wo[2];
#pragma unroll
      for (int part = 0; part < 2; ++part) {
        const int pair = lane + 32 * part;
        float sn, cs;
        __sincosf(clock_phase(lam, pair), &sn, &cs);
        const float a = bt * atom_scale(pair);
        wo[part] = pack_bf16(a * cs, -a * sn);
      }
      uint32_t* wrow = reinterpret_cast<uint32_t*>(p.w + row * 128);
      wrow[lane] = wo[0];
      wrow[lane + 32] = wo[1];
    }
    sc_cur = sc_next;
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
}

struct TokenBwdParams {
  const __nv_bfloat16* q;   // [B,T,H,K]
  const __nv_bfloat16* k;
  const float* qw;
  const float* kw;
  const float* q_rs;        // [B,H,TP]
  const float* k_rs;
  const void* dqn;          // [B,H,TP,K] gradient of the normalised q (fp32 or bf16)
  const void* dkn;
  const float* lam;         // [B,H,TP]
  const float* beta_h;
  const void* dw;           // [B,H,TP,128] gradient of the write vector (fp32 or bf16)
  const void* dw_b;         // second term of the write-vector gradient, or null
  __nv_bfloat16* dq;        // [B,T,H,K]
  __nv_bfloat16* dk;
  float* dqw_part;          // [gridDim.x, K]
  float* dkw_part;
  float* dlam;              // [B,H,TP] (phase part, added to by the readout part)
  float* dbeta;             // [B,H,TP]
  int B, T, H, TP;
  long long q_stride, k_stride, dq_stride, dk_stride;  // token strides (elements)
};

// 8 warps per block; warp w of block b handles rows (b*8 + w) + i*gridDim.x*8.
// Each block writes one row of norm-weight partial sums (its rows, fixed order),
// so the partial matrices have gridDim.x rows.
template <int E, typename GT>
__device__ __forceinline__ void load_grad_vec(const void* base, size_t off, float* f) {
  if constexpr (sizeof(GT) == 4)
    load_f32_vec<E>(static_cast<const float*>(base) + off, f);
  else
    load_bf16_vec<E>(static_cast<const __nv_bfloat16*>(base) + off, f);
}
template <typename GT>
__device__ __forceinline__ float2 load_grad_pair(const void* base, size_t off) {
  if constexpr (sizeof(GT) == 4)
    return *reinterpret_cast<const float2*>(static_cast<const float*>(base) + off);
  else
    return __bfloat1622float2(
        *reinterpret_cast<const __nv_bfloat162*>(static_cast<const __nv_bfloat16*>(base) + off));
}

// E consecutive elements of type T kept packed (as loaded) until they are used,
// so that rows loaded ahead cost E*sizeof(T)/4 registers instead of E.
template <int E, typename T>
struct RawVec {
  static constexpr int N = E * int(sizeof(T)) / 4;
  uint32_t w[N];
  __device__ __forceinline__ void load(const T* p) {
    if constexpr (N % 4 == 0) {
#pragma unroll
      for (int i = 0; i < N / 4; ++i) {
        const uint4 v = reinterpret_cast<const uint4*>(p)[i];
        w[4 * i] = v.x, w[4 * i + 1] = v.y, w[4 * i + 2] = v.z, w[4 * i + 3] = v.w;
      }
    } else {
      const uint2 v = *reinterpret_cast<const uint2*>(p);
      w[0] = v.x, w[1] = v.y;
    }
  }
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int i = 0; i < N; ++i) w[i] = 0u;
  }
  __device__ __forceinline__ void unpack(float* f) const {
#pragma unroll
    for (int i = 0; i < N; ++i) {
      if constexpr (sizeof(T) == 4) {
        f[i] = __uint_as_float(w[i]);
      } else {
        f[2 * i] = __uint_as_float(w[i] << 16);
        f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
      }
    }
  }
};

// GT: element type of the incoming gradients (dqn, dkn, dw, dw_b).
// One warp per row (q side, k side and the write-vector adjoint together, so all
// warps carry the same work), every load of the row issued before any
// arithmetic.  Warp w of block b handles rows b*8 + w + i*gridDim.x*8; each block
// writes one row of q and k norm-weight partials (its rows, fixed order), so the
// partial matrices have gridDim.x rows.
template <int K, typename GT>
__global__ void __launch_bounds__(256, 3) token_bwd_kernel(TokenBwdParams p) {
  pdl_wait();
  pdl_trigger();
  constexpr int E = K / 32;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  __shared__ float wts[2][K];
  __shared__ float part_s[2][8][K];
  for (int i = threadIdx.x; i < K; i += 256) {
    wts[0][i] = p.qw[i];
    wts[1][i] = p.kw[i];
  }
  __syncthreads();
  float acc_q[E], acc_k[E];
#pragma unroll
  for (int j = 0; j < E; ++j) acc_q[j] = acc_k[j] = 0.f;
  const size_t rows = size_t(p.B) * p.H * p.TP;
  for (size_t row = size_t(blockIdx.x) * 8 + wid; row < rows; row += size_t(gridDim.x) * 8) {
    const int t = int(row % p.TP);
    const size_t bh = row / p.TP;
    const int b = int(bh / p.H), h = int(bh % p.H);
    const bool real = t < p.T;
    const size_t tok = size_t(b) * p.T + t, col = size_t(h) * K + lane * E;
    RawVec<E, __nv_bfloat16> xq, xk;
    RawVec<E, GT> gq, gk;
    xq.zero(), xk.zero(), gq.zero(), gk.zero();
    float rq = 0.f, rk = 0.f;
    if (real) {
      xq.load(p.q + tok * p.q_stride + col);
      xk.load(p.k + tok * p.k_stride + col);
      gq.load(static_cast<const GT*>(p.dqn) + row * K + lane * E);
      gk.load(static_cast<const GT*>(p.dkn) + row * K + lane * E);
      rq = p.q_rs[row];
      rk = p.k_rs[row];
    }
    const float lam = p.lam[row], bt = p.beta_h[row];
    float2 dwp[2];
#pragma unroll
    for (int part = 0; part < 2; ++part) {
      const int pair = lane + 32 * part;
      dwp[part] = load_grad_pair<GT>(p.dw, row * 128 + 2 * pair);
      if (p.dw_b) {
        const float2 e2 = load_grad_pair<GT>(p.dw_b, row * 128 + 2 * pair);
        dwp[part].x += e2.x;
        dwp[part].y += e2.y;
      }
    }
    // RMSNorm adjoints (ops/qk_norm.py:109-165) of q and k and the write-vector
    // adjoint (ops/utils.py:598-616): the four row sums are reduced together
    float xq_[E], gq_[E], xk_[E], gk_[E];
    xq.unpack(xq_), gq.unpack(gq_), xk.unpack(xk_), gk.unpack(gk_);
    float dotq = 0.f, dotk = 0.f;
#pragma unroll
    for (int j = 0; j < E; j += 4) {
      const float4 wq4 = *reinterpret_cast<const float4*>(&wts[0][lane * E + j]);
      const float4 wk4 = *reinterpret_cast<const float4*>(&wts[1][lane * E + j]);
      const float wq[4] = {wq4.x, wq4.y, wq4.z, wq4.w}, wk[4] = {wk4.x, wk4.y, wk4.z, wk4.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        dotq += gq_[j + i] * wq[i] * xq_[j + i];
        dotk += gk_[j + i] * wk[i] * xk_[j + i];
      }
    }
    float dl = 0.f, db = 0.f;
#pragma unroll
    for (int part = 0; part < 2; ++part) {
      const int pair = lane + 32 * part;
      float sn, cs;
      __sincosf(clock_phase(lam, pair), &sn, &cs);
      const float sc = atom_scale(pair);
      const float de = dwp[part].x, dd = dwp[part].y;
      db += de * sc * cs - dd * sc * sn;
      dl += (-de * bt * sc * sn - dd * bt * sc * cs) * (pair * kTwoPiOver127);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      dotq += __shfl_xor_sync(0xffffffffu, dotq, o);
      dotk += __shfl_xor_sync(0xffffffffu, dotk, o);
      dl += __shfl_xor_sync(0xffffffffu, dl, o);
      db += __shfl_xor_sync(0xffffffffu, db, o);
    }
    dotq *= rq * rq / K;
    dotk *= rk * rk / K;
    float oq[E], ok[E];
#pragma unroll
    for (int j = 0; j < E; ++j) {
      const float wq = wts[0][lane * E + j], wk = wts[1][lane * E + j];
      oq[j] = (gq_[j] * wq - xq_[j] * dotq) * rq;
      ok[j] = (gk_[j] * wk - xk_[j] * dotk) * rk;
      acc_q[j] += xq_[j] * rq * gq_[j];
      acc_k[j] += xk_[j] * rk * gk_[j];
    }
    if (real) {
      store_bf16_vec<E>(p.dq + tok * p.dq_stride + col, oq);
      store_bf16_vec<E>(p.dk + tok * p.dk_stride + col, ok);
    }
    if (lane == 0) {
      p.dlam[row] = dl;
      p.dbeta[row] = db;
    }
  }
#pragma unroll
  for (int j = 0; j < E; ++j) {
    part_s[0][wid][lane * E + j] = acc_q[j];
    part_s[1][wid][lane * E + j] = acc_k[j];
  }
  __syncthreads();
  for (int d = threadIdx.x; d < K; d += 256) {
    float sq = 0.f, sk = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      sq += part_s[0][i][d];
      sk += part_s[1][i][d];
    }
    p.dqw_part[size_t(blockIdx.x) * K + d] = sq;
    p.dkw_part[size_t(blockIdx.x) * K + d] = sk;
  }
}

// TMA-streamed token_bwd for bf16 incoming gradients: persistent CTAs take
// 32-token tiles of one (b, h); warp 8 (one lane) loads the tile's q, k (public
// layout, 3-D maps), dqn, dkn, dw and dw_b rows (head-major, 2-D maps) into a
// two-stage shared ring; warps 0-7 take four tokens each.  Same arithmetic as
// token_bwd_kernel; each CTA writes one row of norm-weight partials (gridDim.x rows).
constexpr int kTbRows = 32;
constexpr int kTbStages = 2;

template <int K>
constexpr int token_bwd_tma_stage() {
  return kTbRows * (4 * K + 2 * 128) * 2;  // q | k | dqn | dkn | dw | dw_b
}
template <int K>
constexpr int token_bwd_tma_smem() {
  return kTbStages * token_bwd_tma_stage<K>() + 1024;
}

template <int K>
__global__ void __launch_bounds__(288, 1)
    token_bwd_tma_kernel(const __grid_constant__ CUtensorMap map_q,
                         const __grid_constant__ CUtensorMap map_k,
                         const __grid_constant__ CUtensorMap map_dqn,
                         const __grid_constant__ CUtensorMap map_dkn,
                         const __grid_constant__ CUtensorMap map_dw,
                         const __grid_constant__ CUtensorMap map_dwb, TokenBwdParams p) {
  constexpr int E = K / 32;
  constexpr int kT = kTbRows * K * 2, kW = kTbRows * 128 * 2;
  constexpr int oQ = 0, oK = kT, oDQ = 2 * kT, oDK = 3 * kT, oDW = 4 * kT, oDWB = 4 * kT + kW;
  constexpr int kStage = token_bwd_tma_stage<K>();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[kTbStages], empty[kTbStages];
  __shared__ int s_abort;
  __shared__ float part_s[2][8][K];
  volatile int* abort_flag = &s_abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = p.TP / kTbRows, ntiles = p.B * p.H * nb;
  const bool has_b = p.dw_b != nullptr;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kTbStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 8);
    }
    s_abort = 0;
    mbar_fence_init();
    prefetch_tmap(&map_q);
    prefetch_tmap(&map_k);
    prefetch_tmap(&map_dqn);
    prefetch_tmap(&map_dkn);
    prefetch_tmap(&map_dw);
    if (has_b) prefetch_tmap(&map_dwb);
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();
  float acc_q[E], acc_k[E];
#pragma unroll
  for (int j = 0; j < E; ++j) acc_q[j] = acc_k[j] = 0.f;
  if (warp == 8) {
    if (lane == 0) {
      int issued = 0;
      for (int i = 0, k = blockIdx.x; k < ntiles; ++i, k += gridDim.x) {
        const int s = i % kTbStages;
        if (i >= kTbStages && !mbar_wait(&empty[s], ((i / kTbStages) - 1) & 1)) {
          *abort_flag = 1;
          break;
        }
        const int bh = k / nb, t0 = (k % nb) * kTbRows, row0 = bh * p.TP + t0;
        uint8_t* st = smem + s * kStage;
        mbar_expect_tx(&full[s], 4 * kT + (has_b ? 2 : 1) * kW);
        tma_load_3d(st + oQ, &map_q, &full[s], (bh % p.H) * K, t0, bh / p.H);
        tma_load_3d(st + oK, &map_k, &full[s], (bh % p.H) * K, t0, bh / p.H);
        tma_load_2d(st + oDQ, &map_dqn, &full[s], 0, row0);
        tma_load_2d(st + oDK, &map_dkn, &full[s], 0, row0);
        tma_load_2d(st + oDW, &map_dw, &full[s], 0, row0);
        if (has_b) tma_load_2d(st + oDWB, &map_dwb, &full[s], 0, row0);
        issued = i + 1;
      }
      for (int i = issued > kTbStages ? issued - kTbStages : 0; i < issued; ++i)
        mbar_wait(&full[i % kTbStages], (i / kTbStages) & 1);
    }
  } else {
    float wq[E], wk[E];
    load_f32_vec<E>(p.qw + lane * E, wq);
    load_f32_vec<E>(p.kw + lane * E, wk);
    const int r0 = warp * 4;
    // q_rs, k_rs, lam, beta of the warp's four rows (lanes 0-3), one tile ahead
    auto scal = [&](int k) {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (lane < 4 && k < ntiles) {
        const size_t row = size_t(k / nb) * p.TP + (k % nb) * kTbRows + r0 + lane;
        v = make_float4(p.q_rs[row], p.k_rs[row], p.lam[row], p.beta_h[row]);
      }
      return v;
    };
    float4 sc_cur = scal(blockIdx.x);
    for (int i = 0, k = blockIdx.x; k < ntiles; ++i, k += gridDim.x) {
      const float4 sc_next = scal(k + gridDim.x);
      const int s = i % kTbStages;
      const bool got = __all_sync(0xffffffffu, *abort_flag == 0 &&
                                                   mbar_wait(&full[s], (i / kTbStages) & 1));
      if (!got) {
        *abort_flag = 1;
        break;
      }
      const int bh = k / nb, t0 = (k % nb) * kTbRows;
      const int b = bh / p.H, h = bh % p.H;
      const uint8_t* st = smem + s * kStage;
#pragma unroll 1
      for (int u = 0; u < 4; ++u) {
        const int t = t0 + r0 + u;
        const bool real = t < p.T;
        const size_t row = size_t(bh) * p.TP + t;
        const float rq = __shfl_sync(0xffffffffu, sc_cur.x, u);
        const float rk = __shfl_sync(0xffffffffu, sc_cur.y, u);
        const float lam = __shfl_sync(0xffffffffu, sc_cur.z, u);
        const float bt = __shfl_sync(0xffffffffu, sc_cur.w, u);
        const int off = (r0 + u) * K * 2 + lane * E * 2;
        float xq_[E], gq_[E], xk_[E], gk_[E];
        load_bf16_vec<E>(reinterpret_cast<const __nv_bfloat16*>(st + oQ + off), xq_);
        load_bf16_vec<E>(reinterpret_cast<const __nv_bfloat16*>(st + oK + off), xk_);
        load_bf16_vec<E>(reinterpret_cast<const __nv_bfloat16*>(st + oDQ + off), gq_);
        load_bf16_vec<E>(reinterpret_cast<const __nv_bfloat16*>(st + oDK + off), gk_);
        float dotq = 0.f, dotk = 0.f;
#pragma unroll
        for (int j = 0; j < E; ++j) {
          dotq += gq_[j] * wq[j] * xq_[j];
          dotk += gk_[j] * wk[j] * xk_[j];
        }
        // write-vector adjoint (ops/utils.py:598-616) of dw + dw_b
        float dl = 0.f, db = 0.f;
#pragma unroll
        for (int part = 0; part < 2; ++part) {
          const int pair = lane + 32 * part;
          const int woff = (r0 + u) * 256 + pair * 4;
          float2 dwp = __bfloat1622float2(
              *reinterpret_cast<const __nv_bfloat162*>(st + oDW + woff));
          if (has_b) {
            const float2 e2 = __bfloat1622float2(
                *reinterpret_cast<const __nv_bfloat162*>(st + oDWB + woff));
            dwp.x += e2.x;
            dwp.y += e2.y;
          }
          float sn, cs;
          __sincosf(clock_phase(lam, pair), &sn, &cs);
          const float sc = atom_scale(pair);
          db += dwp.x * sc * cs - dwp.y * sc * sn;
          dl += (-dwp.x * bt * sc * sn - dwp.y * bt * sc * cs) * (pair * kTwoPiOver127);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          dotq += __shfl_xor_sync(0xffffffffu, dotq, o);
          dotk += __shfl_xor_sync(0xffffffffu, dotk, o);
          dl += __shfl_xor_sync(0xffffffffu, dl, o);
          db += __shfl_xor_sync(0xffffffffu, db, o);
        }
        dotq *= rq * rq / K;
        dotk *= rk * rk / K;
        float oq[E], ok[E];
#pragma unroll
        for (int j = 0; j < E; ++j) {
          oq[j] = (gq_[j] * wq[j] - xq_[j] * dotq) * rq;
          ok[j] = (gk_[j] * wk[j] - xk_[j] * dotk) * rk;
          acc_q[j] += xq_[j] * rq * gq_[j];
          acc_k[j] += xk_[j] * rk * gk_[j];
        }
        if (real) {
          const size_t tok = size_t(b) * p.T + t, col = size_t(h) * K + lane * E;
          store_bf16_vec<E>(p.dq + tok * p.dq_stride + col, oq);
          store_bf16_vec<E>(p.dk + tok * p.dk_stride + col, ok);
        }
        if (lane == 0) {
          p.dlam[row] = dl;
          p.dbeta[row] = db;
        }
      }
      sc_cur = sc_next;
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
  }
  if (warp < 8) {
#pragma unroll
    for (int j = 0; j < E; ++j) {
      part_s[0][warp][lane * E + j] = acc_q[j];
      part_s[1][warp][lane * E + j] = acc_k[j];
    }
  }
  __syncthreads();
  for (int d = threadIdx.x; d < K; d += blockDim.x) {
    float sq = 0.f, sk = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      sq += part_s[0][i][d];
      sk += part_s[1][i][d];
    }
    p.dqw_part[size_t(blockIdx.x) * K + d] = sq;
    p.dkw_part[size_t(blockIdx.x) * K + d] = sk;
  }
}

// Number of blocks (= partial rows) token_bwd_kernel uses for a shape: three per SM.
inline int token_bwd_blocks(size_t rows) {
  const size_t want = (rows + 7) / 8;
  return int(want < 444 ? want : 444);
}


constexpr int kMaxDgSlots = 6;  // row-dot partial slots of dG a launch may sum

struct GatesBwdParams {
  const float* dG;       // [ndg][B,H,TP] gradient of the in-tile gate cumsum (natural log),
                         // as ndg partial slots dg_stride elements apart, summed in order
  int ndg;
  long long dg_stride;
  const float* dlam;     // [B,H,TP] clock gradient
  const float* dlam2;    // [B,H,TP] second clock gradient term, or null
  const float* bpart1;   // [B*H, NT, nsub1] tile-end gate terms, or null
  const float* bpart2;   // [B*H, NT, nsub2] or null
  int nsub1, nsub2;
  const float* dbeta_h;  // [B,H,TP]
  const float* dclock;   // [B,H] gradient of the final clock, or null
  float* dg;             // [B,T,H]
  float* ddelta;         // [B,T,H]
  float* dbeta;          // [B,T,H]
  float* dclock0;        // [B,H] or null
  int B, T, H, TP;
  const int* lengths;    // [B] valid tokens (right padding), or null: zero gradients past it
};

// Grid (B*H, ceil(TP/1024)) as the forward: CTA (bh, k) handles token block k,
// and sums the clock-gradient carry from the later blocks itself.
__global__ void __launch_bounds__(1024) gates_bwd_kernel(GatesBwdParams p) {
  pdl_wait();
  pdl_trigger();
  const int bh = blockIdx.x, b = bh / p.H, h = bh % p.H, k = blockIdx.y;
  __shared__ float wsum[32];
  const size_t base = size_t(bh) * p.TP;
  const int t = k * 1024 + threadIdx.x;
  const bool in = t < p.TP;
  auto dlam_at = [&](int tt) {
    if (tt >= p.TP) return 0.f;
    float x = p.dlam[base + tt];
    if (p.dlam2) x += p.dlam2[base + tt];
    return x;
  };
  float v[kMaxDgSlots];
#pragma unroll
  for (int s = 0; s < kMaxDgSlots; ++s)
    v[s] = in && s < p.ndg ? p.dG[s * p.dg_stride + base + t] : 0.f;
  const float dl = dlam_at(t);
  float l[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  const int nblk = gridDim.y;
  int kk = nblk - 1;
  for (; kk - 8 >= k; kk -= 8)
#pragma unroll
    for (int u = 0; u < 8; ++u) l[u] += dlam_at((kk - u) * 1024 + threadIdx.x);
  for (; kk > k; --kk) l[0] += dlam_at(kk * 1024 + threadIdx.x);
  const float later = ((l[0] + l[1]) + (l[2] + l[3])) + ((l[4] + l[5]) + (l[6] + l[7]));
  float dGt = v[0];
#pragma unroll
  for (int s = 1; s < kMaxDgSlots; ++s) dGt += v[s];
  if (in && (t & 127) == 127) {
    const size_t tile = size_t(bh) * (p.TP / 128) + t / 128;
    if (p.bpart1)
      for (int i = 0; i < p.nsub1; ++i) dGt += p.bpart1[tile * p.nsub1 + i];
    if (p.bpart2)
      for (int i = 0; i < p.nsub2; ++i) dGt += p.bpart2[tile * p.nsub2 + i];
  }
  float tot, ltot;
  const ScanPair gs = scan1024<true>(dGt, wsum, &tot);
  const ScanPair ls = scan1024<true>(dl, wsum, &tot);
  scan1024<true>(later, wsum, &ltot);
  const float carry = __fadd_rn(p.dclock ? p.dclock[bh] : 0.f, ltot);
  if (t < p.T) {
    // inputs past a sequence's length were replaced by neutral values: no gradient
    const bool valid = !p.lengths || t < p.lengths[b];
    const size_t i = (size_t(b) * p.T + t) * p.H + h;
    p.dg[i] = valid ? gs.tile : 0.f;
    p.ddelta[i] = valid ? __fadd_rn(carry, ls.block) : 0.f;
    p.dbeta[i] = valid ? p.dbeta_h[base + t] : 0.f;
  }
  if (k == 0 && threadIdx.x == 0 && p.dclock0) p.dclock0[bh] = __fadd_rn(carry, tot);
}

}  // namespace cyfa
