// C-ABI of the chunked op: the layout of the caller-owned saved/work buffers,
// tensor maps, and the launch sequence of the forward (and backward) pass.
#include "../../include/cyfa.h"
#include "cyfa_common.cuh"

namespace cyfa {

// Carves 256-byte aligned sub-buffers out of a caller-owned region.
struct Carver {
  uint8_t* base;
  size_t off = 0;
  explicit Carver(void* b) : base(static_cast<uint8_t*>(b)) {}
  template <typename T>
  T* take(size_t count) {
    off = (off + 255) / 256 * 256;
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += count * sizeof(T);
    return p;
  }
};

struct Dims {
  int B, T, H, K, V, TP, NT, BH;
};

static Dims make_dims(int B, int T, int H, int K, int V) {
  Dims d{B, T, H, K, V, 0, 0, B * H};
  d.TP = (T + 127) / 128 * 128;
  d.NT = d.TP / 128;
  return d;
}

// Tensors the forward pass keeps for the backward pass.
struct Saved {
  float *G, *lam, *beta_h, *q_rs, *k_rs;
  __nv_bfloat16 *qn, *kn, *w, *raw, *weights, *s1, *s2;
};

static Saved carve_saved(const Dims& d, void* base, size_t* total) {
  Carver c(base);
  Saved s;
  const size_t n = size_t(d.BH) * d.TP;
  s.G = c.take<float>(n);
  s.lam = c.take<float>(n);
  s.beta_h = c.take<float>(n);
  s.q_rs = c.take<float>(n);
  s.k_rs = c.take<float>(n);
  s.qn = c.take<__nv_bfloat16>(n * d.K);
  s.kn = c.take<__nv_bfloat16>(n * d.K);
  s.w = c.take<__nv_bfloat16>(n * 128);
  s.raw = c.take<__nv_bfloat16>(n * 128);
  s.weights = c.take<__nv_bfloat16>(n * 128);
  s.s1 = c.take<__nv_bfloat16>(size_t(d.BH) * d.NT * d.K * 128);
  s.s2 = c.take<__nv_bfloat16>(size_t(d.BH) * d.NT * 128 * d.V);
  if (total) *total = c.off + 256;
  return s;
}

// [B,T,H,D] bf16 as the 4-D map {D, H, T, B} with a {64, 1, 128, 1} box.
static int tmap_public(CUtensorMap* m, const void* base, int B, int T, int H, int D) {
  const uint64_t dims[4] = {uint64_t(D), uint64_t(H), uint64_t(T), uint64_t(B)};
  const uint64_t strides[3] = {uint64_t(D) * 2, uint64_t(H) * D * 2, uint64_t(T) * H * D * 2};
  const uint32_t box[4] = {64, 1, 128, 1};
  return make_tmap_bf16(m, base, 4, dims, strides, box);
}

static bool shape_ok(int B, int T, int H, int K, int V) {
  return B > 0 && T > 0 && H > 0 && (K == 128 || K == 256) && (V == 128 || V == 256) &&
         size_t(B) * H * ((T + 127) / 128 * 128) < (size_t(1) << 31);
}

template <typename Kern>
static void set_smem(Kern k, int bytes) {
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

}  // namespace cyfa

using namespace cyfa;

extern "C" {

size_t cyfa_chunk_saved_bytes(int B, int T, int H, int K, int V) {
  if (!shape_ok(B, T, H, K, V)) return 0;
  size_t total = 0;
  carve_saved(make_dims(B, T, H, K, V), nullptr, &total);
  return total;
}

int cyfa_chunk_fwd(const cyfa_chunk_fwd_args* a, void* saved, size_t saved_bytes, void* stream) {
  CYFA_REQUIRE(a && saved, kNullPointer);
  CYFA_REQUIRE(shape_ok(a->B, a->T, a->H, a->K, a->V), kBadShape);
  CYFA_REQUIRE(a->q && a->k && a->v && a->g && a->delta && a->beta && a->q_norm_weight &&
                   a->k_norm_weight && a->table_bf && a->o && a->hk && a->hv && a->clock,
               kNullPointer);
  const Dims d = make_dims(a->B, a->T, a->H, a->K, a->V);
  size_t need = 0;
  carve_saved(d, nullptr, &need);
  CYFA_REQUIRE(saved_bytes >= need, kWorkspace);
  CYFA_REQUIRE(aligned(saved, 256), kMisaligned);
  CYFA_REQUIRE(aligned(a->q, 16) && aligned(a->k, 16) && aligned(a->v, 16) && aligned(a->o, 16) &&
                   aligned(a->hk, 16) && aligned(a->hv, 16) && aligned(a->table_bf, 16) &&
                   (!a->hk0 || aligned(a->hk0, 16)) && (!a->hv0 || aligned(a->hv0, 16)),
               kMisaligned);
  const Saved s = carve_saved(d, saved, nullptr);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc;

  rc = cyfa_gates_fwd(a->g, a->delta, a->beta, a->clock0, s.G, s.lam, s.beta_h, a->clock, d.B,
                      d.T, d.H, stream);
  if (rc) return rc;
  rc = cyfa_token_fwd(a->q, a->k, a->q_norm_weight, a->k_norm_weight, s.lam, s.beta_h, s.qn, s.kn,
                      s.w, s.q_rs, s.k_rs, d.B, d.T, d.H, d.K, a->q_eps, a->k_eps, stream);
  if (rc) return rc;

  const uint64_t rows = uint64_t(d.BH) * d.TP;
  CUtensorMap m_qn, m_kn, m_w, m_v, m_s1, m_s2, m_tab, m_weights;
  if ((rc = tmap_2d(&m_qn, s.qn, rows, d.K, 128))) return rc;
  if ((rc = tmap_2d(&m_kn, s.kn, rows, d.K, 128))) return rc;
  if ((rc = tmap_2d(&m_w, s.w, rows, 128, 128))) return rc;
  if ((rc = tmap_2d(&m_weights, s.weights, rows, 128, 128))) return rc;
  if ((rc = tmap_public(&m_v, a->v, d.B, d.T, d.H, d.V))) return rc;
  if ((rc = tmap_2d(&m_s1, s.s1, uint64_t(d.BH) * d.NT * d.K, 128, d.K))) return rc;
  if ((rc = tmap_2d(&m_s2, s.s2, uint64_t(d.BH) * d.NT * 128, d.V, 128))) return rc;
  if ((rc = tmap_2d(&m_tab, a->table_bf, uint64_t(d.H) * 128, 128, 128))) return rc;

  // ---- pass 1: key memory (k^, w) -> raw, then the readout -> weights
  {
    ScanParams p{d.BH, d.H, d.TP, d.NT, d.K, 128, kRows2D, kRows2D, s.G, a->hk0, s.s1, a->hk,
                 0.f, nullptr, nullptr, nullptr};
    set_smem(state_scan_kernel<false>, kScanSmem);
    state_scan_kernel<false><<<dim3(d.BH, d.K / 128, 2), 128, kScanSmem, st>>>(m_kn, m_w, p);
    if ((rc = launch_status())) return rc;
    TileFwdParams t{d.BH, d.H, d.TP, d.NT, d.T, 128, kRows2D, 0, s.G, s.lam, a->scale, s.raw,
                    s.weights};
    if (d.K == 256) {
      set_smem(tile_fwd_kernel<256, true>, tile_fwd_smem<256>());
      tile_fwd_kernel<256, true><<<dim3(d.BH * d.NT, 1), 128, tile_fwd_smem<256>(), st>>>(
          m_qn, m_kn, m_w, m_s1, m_tab, t);
    } else {
      set_smem(tile_fwd_kernel<128, true>, tile_fwd_smem<128>());
      tile_fwd_kernel<128, true><<<dim3(d.BH * d.NT, 1), 128, tile_fwd_smem<128>(), st>>>(
          m_qn, m_kn, m_w, m_s1, m_tab, t);
    }
    if ((rc = launch_status())) return rc;
  }
  // ---- pass 2: value memory (weights as queries, w as keys, v) -> o
  {
    ScanParams p{d.BH, d.H, d.TP, d.NT, 128, d.V, kRows2D, kPublic4D, s.G, a->hv0, s.s2, a->hv,
                 0.f, nullptr, nullptr, nullptr};
    state_scan_kernel<false><<<dim3(d.BH, 1, d.V / 64), 128, kScanSmem, st>>>(m_w, m_v, p);
    if ((rc = launch_status())) return rc;
    TileFwdParams t{d.BH, d.H, d.TP, d.NT, d.T, d.V, kPublic4D, 1, s.G, s.lam, 1.f,
                    static_cast<__nv_bfloat16*>(a->o), nullptr};
    set_smem(tile_fwd_kernel<128, false>, tile_fwd_smem<128>());
    tile_fwd_kernel<128, false><<<dim3(d.BH * d.NT, d.V / 128), 128, tile_fwd_smem<128>(), st>>>(
        m_weights, m_w, m_v, m_s2, m_tab, t);
    if ((rc = launch_status())) return rc;
  }
  return kOk;
}

}  // extern "C"
