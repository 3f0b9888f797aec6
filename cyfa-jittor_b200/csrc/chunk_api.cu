// C-ABI of the chunked op: the layout of the caller-owned saved/work buffers,
// tensor maps, and the launch sequence of the forward (and backward) pass.
#include <mutex>
#include <set>
#include <tuple>

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

// Segments of a state scan: when a scan has fewer CTAs than the SMs (few
// sequences x heads, long sequences), its tiles are split
// into segments scanned side by side (a summary pass from zero, the carries, and
// the real pass from the carried states), at least 16 tiles each, so that the
// two extra launches pay off against the serial chain they shorten.
// Tiles per segment; the segments are ceil(NT / that), none empty.
static int scan_seg_tiles(const Dims& d, int ctas) {
  if (!g_scan_split.load(std::memory_order_relaxed)) return d.NT;
  int n = 148 / (ctas > 0 ? ctas : 1);
  const int cap = d.NT / 16;
  if (n > cap) n = cap;
  if (n > kScanCarryMaxSegs) n = kScanCarryMaxSegs;
  return n < 2 ? d.NT : (d.NT + n - 1) / n;
}
static int scan_nseg(const Dims& d, int ctas) {
  const int per = scan_seg_tiles(d, ctas);
  return (d.NT + per - 1) / per;
}

// fp32 scratch of the segmented scans: segment end states and carried states,
// [nseg, BH, DK, DV] each, for the larger of the two passes.
static size_t scan_scratch_floats(const Dims& d) {
  const int n1 = scan_nseg(d, d.BH * (d.K / 128) * 2), n2 = scan_nseg(d, d.BH * (d.V / 64));
  const int n = n1 > n2 ? n1 : n2;
  const size_t elems = size_t(d.K) * 128 > size_t(128) * d.V ? size_t(d.K) * 128 : size_t(128) * d.V;
  return n > 1 ? 2 * size_t(n) * d.BH * elems : 0;
}

// Tensors the forward pass keeps for the backward pass.
struct Saved {
  float *G, *lam, *beta_h, *q_rs, *k_rs;
  __nv_bfloat16 *qn, *kn, *w, *raw, *weights, *s1, *s2;
  __nv_bfloat16 *s1_fin, *s2_fin;  // bf16 copies of the final states (reverse boundary terms)
  float* scan_tmp;                 // segmented-scan scratch (scan_scratch_floats)
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
  s.s1_fin = c.take<__nv_bfloat16>(size_t(d.BH) * d.K * 128);
  s.s2_fin = c.take<__nv_bfloat16>(size_t(d.BH) * 128 * d.V);
  s.scan_tmp = c.take<float>(scan_scratch_floats(d));
  if (total) *total = c.off + 256;
  return s;
}

// Row-dot slots of dG: dweights, dw, and up to two 128-column blocks each of dq^, dk^.
constexpr int kDgSlots = 6;

// Scratch of the backward pass.
struct Work {
  __nv_bfloat16 *h1, *h2, *A, *Bp, *draw, *dweights, *dw, *dw_b, *dq1, *dk1;
  float *dG, *dlam_r, *dlam_w, *dbeta_h, *bpart1, *bpart2, *dtab_part,
      *dqw_part, *dkw_part, *scan_tmp;
};

static Work carve_work(const Dims& d, void* base, size_t* total) {
  Carver c(base);
  Work w;
  const size_t n = size_t(d.BH) * d.TP, tiles = size_t(d.BH) * d.NT;
  w.h1 = c.take<__nv_bfloat16>(tiles * d.K * 128);
  w.h2 = c.take<__nv_bfloat16>(tiles * 128 * d.V);
  w.A = c.take<__nv_bfloat16>(tiles * 128 * 128);
  w.Bp = c.take<__nv_bfloat16>(tiles * 128 * 128);
  w.draw = c.take<__nv_bfloat16>(n * 128);
  w.dweights = c.take<__nv_bfloat16>(n * 128);
  w.dw = c.take<__nv_bfloat16>(n * 128);
  w.dw_b = c.take<__nv_bfloat16>(n * 128);
  w.dq1 = c.take<__nv_bfloat16>(n * d.K);
  w.dk1 = c.take<__nv_bfloat16>(n * d.K);
  w.dG = c.take<float>(n * kDgSlots);
  w.dlam_r = c.take<float>(n);
  w.dlam_w = c.take<float>(n);
  w.dbeta_h = c.take<float>(n);
  w.bpart1 = c.take<float>(tiles * (d.K / 128) * 2 * 4);
  w.bpart2 = c.take<float>(tiles * (d.V / 64) * 4);
  w.dtab_part = c.take<float>(tiles * 128 * 128);
  w.dqw_part = c.take<float>(size_t(1184) * d.K);
  w.dkw_part = c.take<float>(size_t(1184) * d.K);
  w.scan_tmp = c.take<float>(scan_scratch_floats(d));
  if (total) *total = c.off + 256;
  return w;
}

// [B,T,H,D] bf16 whose tokens are `stride` elements apart (stride >= H*D) as the
// 4-D map {D, H, T, B} with a {64, 1, 128, 1} box.
static int tmap_public(CUtensorMap* m, const void* base, int B, int T, int H, int D,
                       long long stride, uint32_t box_rows = 128) {
  const uint64_t dims[4] = {uint64_t(D), uint64_t(H), uint64_t(T), uint64_t(B)};
  const uint64_t strides[3] = {uint64_t(D) * 2, uint64_t(stride) * 2,
                               uint64_t(T) * uint64_t(stride) * 2};
  const uint32_t box[4] = {64, 1, box_rows, 1};
  return make_tmap_bf16(m, base, 4, dims, strides, box);
}

static bool shape_ok(int B, int T, int H, int K, int V) {
  return B > 0 && T > 0 && H > 0 && (K == 128 || K == 256) && (V == 128 || V == 256) &&
         size_t(B) * H * ((T + 127) / 128 * 128) < (size_t(1) << 31);
}

// Token strides must be 0 (dense) or at least the row width and a multiple of 8
// elements (16 bytes, the TMA stride rule).
static bool strides_ok(long long s, long long dense) { return s == 0 || (s >= dense && s % 8 == 0); }

// CTAs per head of the persistent readout adjoint: about one CTA per SM in
// total, at least one tile each.
static int readout_ctas_per_head(const Dims& d) {
  const int want = (148 + d.H - 1) / d.H;
  const int tiles = d.B * d.NT;
  return want < tiles ? want : tiles;
}

// A token stride of 0 means the dense layout.
static long long stride_or(long long s, long long dense) { return s > 0 ? s : dense; }

// One state scan over grid (BH, K slices, V slices): a single launch, or, with
// scan_nseg segments, the summary pass, the carries and the segmented pass
// (state_scan_kernel, scan_carry_kernel).  `tmp`: scan_scratch_floats floats.
template <bool REVERSE>
static int run_scan(const Dims& d, ScanParams p, dim3 grid, const CUtensorMap& mk,
                    const CUtensorMap& mv, const CUtensorMap& mf, const CUtensorMap& mff,
                    float* tmp, cudaStream_t st) {
  const char* name = REVERSE ? "state_scan_bwd" : "state_scan_fwd";
  const int ctas = int(grid.x * grid.y * grid.z);
  const int nseg = scan_nseg(d, ctas);
  p.nseg = nseg;
  p.seg_tiles = scan_seg_tiles(d, ctas);
  p.summary = 0;
  set_smem(state_scan_kernel<REVERSE>, kScanSmem);
  if (nseg == 1) {
    CYFA_LAUNCH(name, st, (launch_k(state_scan_kernel<REVERSE>, grid, kScanThreads, kScanSmem,
                                    st, mk, mv, mf, mff, p)));
    return launch_status();
  }
  CYFA_REQUIRE(tmp, kWorkspace);
  const size_t elems = size_t(p.DK) * p.DV;
  float* seg_out = tmp;
  float* seg_init = tmp + size_t(nseg) * d.BH * elems;
  const dim3 sgrid(grid.x, grid.y, grid.z * nseg);
  ScanParams a = p;
  a.summary = 1;
  a.seg_out = seg_out;
  CYFA_LAUNCH("state_scan_summary", st,
              (launch_k(state_scan_kernel<REVERSE>, sgrid, kScanThreads, kScanSmem, st, mk, mv,
                        mf, mff, a)));
  int rc = launch_status();
  if (rc) return rc;
  const int e = int(elems);
  CYFA_LAUNCH("scan_carry", st,
              (launch_k(scan_carry_kernel<REVERSE>, dim3((e / 4 + 255) / 256, d.BH), 256, 0, st,
                        static_cast<const float*>(p.G), d.TP, d.NT, d.BH, e, nseg, p.seg_tiles,
                        static_cast<const float*>(seg_out), seg_init)));
  if ((rc = launch_status())) return rc;
  p.seg_init = seg_init;
  CYFA_LAUNCH(name, st, (launch_k(state_scan_kernel<REVERSE>, sgrid, kScanThreads, kScanSmem, st,
                                  mk, mv, mf, mff, p)));
  return launch_status();
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
  CYFA_REQUIRE(strides_ok(a->q_stride, d.H * d.K) && strides_ok(a->k_stride, d.H * d.K) &&
                   strides_ok(a->v_stride, d.H * d.V),
               kBadShape);
  const Saved s = carve_saved(d, saved, nullptr);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc;

  rc = gates_fwd_launch(a->g, a->delta, a->beta, a->clock0, s.G, s.lam, s.beta_h, a->clock, d.B,
                        d.T, d.H, a->lengths, stream);
  if (rc) return rc;
  rc = token_fwd_launch(a->q, a->k, a->q_norm_weight, a->k_norm_weight, s.lam, s.beta_h, s.qn,
                        s.kn, s.w, s.q_rs, s.k_rs, d.B, d.T, d.H, d.K, a->q_eps, a->k_eps,
                        stride_or(a->q_stride, d.H * d.K), stride_or(a->k_stride, d.H * d.K),
                        stream);
  if (rc) return rc;

  const uint64_t rows = uint64_t(d.BH) * d.TP;
  CUtensorMap m_qn, m_kn, m_w, m_v, m_s1, m_s2, m_tab, m_weights;
  if ((rc = tmap_2d(&m_qn, s.qn, rows, d.K, 128))) return rc;
  if ((rc = tmap_2d(&m_kn, s.kn, rows, d.K, 128))) return rc;
  if ((rc = tmap_2d(&m_w, s.w, rows, 128, 128))) return rc;
  if ((rc = tmap_2d(&m_weights, s.weights, rows, 128, 128))) return rc;
  if ((rc = tmap_public(&m_v, a->v, d.B, d.T, d.H, d.V, stride_or(a->v_stride, d.H * d.V))))
    return rc;
  if ((rc = tmap_2d(&m_s1, s.s1, uint64_t(d.BH) * d.NT * d.K, 128, d.K))) return rc;
  if ((rc = tmap_2d(&m_s2, s.s2, uint64_t(d.BH) * d.NT * 128, d.V, 128))) return rc;
  if ((rc = tmap_2d(&m_tab, a->table_bf, uint64_t(d.H) * 128, 128, 128))) return rc;

  // ---- pass 1: key memory (k^, w) -> raw, then the readout -> weights
  {
    ScanParams p{d.BH, d.H, d.TP, d.NT, d.K, 128, kRows2D, kRows2D, s.G, a->hk0, s.s1, a->hk,
                 0.f, s.s1_fin, nullptr};
    if ((rc = run_scan<false>(d, p, dim3(d.BH, d.K / 128, 2), m_kn, m_w, m_kn, m_kn, s.scan_tmp,
                              st)))
      return rc;
    TileFwdParams t{d.BH, d.H, d.TP, d.NT, d.T, 128, kRows2D, 0, s.G, s.lam, a->scale, s.raw,
                    s.weights};
    // the state history in 64-row blocks, as the two-CTA kernel streams it
    CUtensorMap m_s1_64;
    if ((rc = tmap_2d(&m_s1_64, s.s1, uint64_t(d.BH) * d.NT * d.K, 128, 64))) return rc;
    if (d.K == 256) {
      set_smem(tile_fwd_ro_kernel<256>, kRoSmem);
      CYFA_LAUNCH("tile_fwd_readout", st,
                  (launch_k(tile_fwd_ro_kernel<256>, dim3(d.BH * d.NT, 1), 256, kRoSmem, st, m_qn,
                            m_kn, m_w, m_s1_64, m_tab, t)));
    } else {
      set_smem(tile_fwd_ro_kernel<128>, kRoSmem);
      CYFA_LAUNCH("tile_fwd_readout", st,
                  (launch_k(tile_fwd_ro_kernel<128>, dim3(d.BH * d.NT, 1), 256, kRoSmem, st, m_qn,
                            m_kn, m_w, m_s1_64, m_tab, t)));
    }
    if ((rc = launch_status())) return rc;
  }
  // ---- pass 2: value memory (weights as queries, w as keys, v) -> o
  {
    ScanParams p{d.BH, d.H, d.TP, d.NT, 128, d.V, kRows2D, kPublic4D, s.G, a->hv0, s.s2, a->hv,
                 0.f, s.s2_fin, nullptr};
    if ((rc = run_scan<false>(d, p, dim3(d.BH, 1, d.V / 64), m_w, m_v, m_w, m_w, s.scan_tmp, st)))
      return rc;
    TileFwdParams t{d.BH, d.H, d.TP, d.NT, d.T, d.V, kPublic4D, 1, s.G, s.lam, 1.f,
                    static_cast<__nv_bfloat16*>(a->o), nullptr};
    set_smem(tile_fwd_kernel, kTileFwdSmem);
    CYFA_LAUNCH("tile_fwd", st,
                (launch_k(tile_fwd_kernel, dim3(d.BH * d.NT, d.V / 128), 256, kTileFwdSmem, st,
                          m_weights, m_w, m_v, m_s2, t)));
    if ((rc = launch_status())) return rc;
  }
  return kOk;
}

int cyfa_readout_table(const float* readout, const float* basis, void* table_bf, int H,
                       void* stream) {
  CYFA_REQUIRE(readout && basis && table_bf, kNullPointer);
  CYFA_REQUIRE(H > 0, kBadShape);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CYFA_LAUNCH("readout_table", st,
              launch_k(readout_table_kernel, dim3(H, 128), 128, 0, st, readout, basis,
                       static_cast<__nv_bfloat16*>(table_bf)));
  return launch_status();
}

int cyfa_readout_table_grad(const float* dtable, const float* basis_t, float* dreadout, int H,
                            void* stream) {
  CYFA_REQUIRE(dtable && basis_t && dreadout, kNullPointer);
  CYFA_REQUIRE(H > 0, kBadShape);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CYFA_LAUNCH("readout_grad", st,
              launch_k(readout_grad_kernel, dim3(H, 127), 128, 0, st, dtable, basis_t, dreadout));
  return launch_status();
}

size_t cyfa_chunk_work_bytes(int B, int T, int H, int K, int V) {
  if (!shape_ok(B, T, H, K, V)) return 0;
  size_t total = 0;
  carve_work(make_dims(B, T, H, K, V), nullptr, &total);
  return total;
}

int cyfa_chunk_bwd(const cyfa_chunk_bwd_args* g, const void* saved, size_t saved_bytes,
                   void* work, size_t work_bytes, void* stream) {
  CYFA_REQUIRE(g && saved && work, kNullPointer);
  const cyfa_chunk_fwd_args* a = &g->fwd;
  CYFA_REQUIRE(shape_ok(a->B, a->T, a->H, a->K, a->V), kBadShape);
  CYFA_REQUIRE(a->q && a->k && a->v && a->q_norm_weight && a->k_norm_weight && a->table_bf &&
                   a->hk && a->hv && g->d_o && g->dq && g->dk && g->dv && g->dg && g->ddelta &&
                   g->dbeta && g->dtable && g->dq_norm_weight && g->dk_norm_weight,
               kNullPointer);
  CYFA_REQUIRE(!g->dreadout || g->readout_basis_t, kNullPointer);
  const Dims d = make_dims(a->B, a->T, a->H, a->K, a->V);
  size_t need_s = 0, need_w = 0;
  carve_saved(d, nullptr, &need_s);
  carve_work(d, nullptr, &need_w);
  CYFA_REQUIRE(saved_bytes >= need_s && work_bytes >= need_w, kWorkspace);
  CYFA_REQUIRE(aligned(saved, 256) && aligned(work, 256), kMisaligned);
  CYFA_REQUIRE(aligned(g->d_o, 16) && aligned(g->dv, 16) && aligned(a->v, 16) &&
                   (!g->dhk || aligned(g->dhk, 16)) && (!g->dhv || aligned(g->dhv, 16)) &&
                   (!g->dhk0 || aligned(g->dhk0, 16)) && (!g->dhv0 || aligned(g->dhv0, 16)),
               kMisaligned);
  CYFA_REQUIRE(strides_ok(a->q_stride, d.H * d.K) && strides_ok(a->k_stride, d.H * d.K) &&
                   strides_ok(a->v_stride, d.H * d.V) && strides_ok(g->dq_stride, d.H * d.K) &&
                   strides_ok(g->dk_stride, d.H * d.K) && strides_ok(g->dv_stride, d.H * d.V),
               kBadShape);
  const Saved s = carve_saved(d, const_cast<void*>(saved), nullptr);
  const Work w = carve_work(d, work, nullptr);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc;
  const uint64_t rows = uint64_t(d.BH) * d.TP, trows = uint64_t(d.BH) * d.NT * 128;
  CUtensorMap m_qn, m_kn, m_w, m_weights, m_v, m_do, m_draw, m_s1, m_s2, m_h1, m_h2, m_A, m_Bp,
      m_tab;
  if ((rc = tmap_2d(&m_qn, s.qn, rows, d.K, 128))) return rc;
  if ((rc = tmap_2d(&m_kn, s.kn, rows, d.K, 128))) return rc;
  if ((rc = tmap_2d(&m_w, s.w, rows, 128, 128))) return rc;
  if ((rc = tmap_2d(&m_weights, s.weights, rows, 128, 128))) return rc;
  if ((rc = tmap_2d(&m_draw, w.draw, rows, 128, 128))) return rc;
  if ((rc = tmap_public(&m_v, a->v, d.B, d.T, d.H, d.V, stride_or(a->v_stride, d.H * d.V))))
    return rc;
  if ((rc = tmap_public(&m_do, g->d_o, d.B, d.T, d.H, d.V, (long long)d.H * d.V))) return rc;
  if ((rc = tmap_2d(&m_s1, s.s1, uint64_t(d.BH) * d.NT * d.K, 128, 128))) return rc;
  if ((rc = tmap_2d(&m_h1, w.h1, uint64_t(d.BH) * d.NT * d.K, 128, 128))) return rc;
  if ((rc = tmap_2d(&m_s2, s.s2, uint64_t(d.BH) * d.NT * 128, d.V, 128))) return rc;
  if ((rc = tmap_2d(&m_h2, w.h2, uint64_t(d.BH) * d.NT * 128, d.V, 128))) return rc;
  if ((rc = tmap_2d(&m_A, w.A, trows, 128, 128))) return rc;
  if ((rc = tmap_2d(&m_Bp, w.Bp, trows, 128, 128))) return rc;
  if ((rc = tmap_2d(&m_tab, a->table_bf, uint64_t(d.H) * 128, 128, 128))) return rc;
  // 64-row boxes: operands the dual GEMM reads MN-major in 64-row k-blocks
  CUtensorMap m_qn64, m_kn64, m_w64, m_weights64, m_do64, m_draw64, m_h1_64, m_h2_64, m_A64,
      m_Bp64;
  if ((rc = tmap_2d(&m_qn64, s.qn, rows, d.K, 64))) return rc;
  if ((rc = tmap_2d(&m_kn64, s.kn, rows, d.K, 64))) return rc;
  if ((rc = tmap_2d(&m_w64, s.w, rows, 128, 64))) return rc;
  if ((rc = tmap_2d(&m_weights64, s.weights, rows, 128, 64))) return rc;
  if ((rc = tmap_2d(&m_draw64, w.draw, rows, 128, 64))) return rc;
  if ((rc = tmap_public(&m_do64, g->d_o, d.B, d.T, d.H, d.V, (long long)d.H * d.V, 64))) return rc;
  if ((rc = tmap_2d(&m_h1_64, w.h1, uint64_t(d.BH) * d.NT * d.K, 128, 64))) return rc;
  if ((rc = tmap_2d(&m_h2_64, w.h2, uint64_t(d.BH) * d.NT * 128, d.V, 64))) return rc;
  if ((rc = tmap_2d(&m_A64, w.A, trows, 128, 64))) return rc;
  if ((rc = tmap_2d(&m_Bp64, w.Bp, trows, 128, 64))) return rc;
  const dim3 tiles(d.BH * d.NT);
  set_smem(state_scan_kernel<true>, kScanSmem);
  set_smem(dual_gemm_kernel, kDualSmem);
  set_smem(tile_scores_kernel, kScoresSmem);
  const unsigned scores_grid = 2 * d.BH * d.NT < 148 ? 2 * d.BH * d.NT : 148;  // persistent
  // The three GEMM pairs of a pass in one persistent launch, their 128-column
  // units interleaved tile by tile.
  auto dual = [&](const DualMaps& m, DualParams& p, int njobs) {
    p.units = 0;
    for (int jx = 0; jx < njobs; ++jx)
      for (int nb = 0; nb < p.job[jx].N / 128; ++nb) {
        p.unit_job[p.units] = jx;
        p.unit_nb[p.units] = nb;
        ++p.units;
      }
    const unsigned nu = unsigned(d.BH * d.NT * p.units), grid = nu < 148 ? nu : 148;
    CYFA_LAUNCH("dual_gemm", st,
                (launch_k(dual_gemm_kernel, grid, kDualThreads, kDualSmem, st, m, p)));
    return launch_status();
  };
  // row-dot slots of dG (summed by gates_bwd): dweights, dw, dq^ blocks, dk^ blocks
  const size_t slot = size_t(d.BH) * d.TP;
  const int ndg = 2 + 2 * (d.K / 128);
  // boundary partials per tile: one per (CTA slice, warp)
  const int nsub1 = (d.K / 128) * 2 * 4, nsub2 = (d.V / 64) * 4;

  // ================= pass 2 (queries = weights, keys = w, values = v)
  {
    ScanParams p{d.BH, d.H, d.TP, d.NT, 128, d.V, kRows2D, kPublic4D, s.G, g->dhv, w.h2, g->dhv0,
                 1.f, nullptr, w.bpart2, a->hv};
    CUtensorMap m_ff2;
    if ((rc = tmap_2d(&m_ff2, s.s2_fin, uint64_t(d.BH) * 128, d.V, 128))) return rc;
    if ((rc = run_scan<true>(d, p, dim3(d.BH, 1, d.V / 64), m_weights, m_do, m_s2, m_ff2,
                             w.scan_tmp, st)))
      return rc;
    ScoresParams sp{d.BH, d.H, d.TP, d.NT, 128, d.V, kPublic4D, kPublic4D, s.G, 1.f, w.A, w.Bp};
    CYFA_LAUNCH("tile_scores", st,
                (launch_k(tile_scores_kernel, scores_grid, kScoresThreads, kScoresSmem, st,
                          m_weights, m_w, m_do, m_v, sp)));
    if ((rc = launch_status())) return rc;
    DualMaps m;
    DualParams dp{d.BH, d.H, d.TP, d.NT, d.T, s.G};
    // dweights = B' w + 2^{G_t} dO S^T ;  dG slot 0 = weights . dweights
    m.x1[0] = m_Bp, m.y1[0] = m_w64, m.x2[0] = m_do, m.y2[0] = m_s2;
    dp.job[0] = DualJob{0, kRows2D, kPublic4D, 1, 128, d.V, 1.f, 0, 3, w.dweights, 0, s.weights,
                        1.f, w.dG};
    // dw = B'^T weights + 2^{G_L-G_s} v H^T ;  dG slot 1 = -(w . dw)
    m.x1[1] = m_Bp64, m.y1[1] = m_weights64, m.x2[1] = m_v, m.y2[1] = m_h2;
    dp.job[1] = DualJob{1, kRows2D, kPublic4D, 1, 128, d.V, 1.f, 1, 3, w.dw, 0, s.w, -1.f,
                        w.dG + slot};
    // dv = A^T dO + 2^{G_L-G_s} w H  (public layout)
    m.x1[2] = m_A64, m.y1[2] = m_do64, m.x2[2] = m_w, m.y2[2] = m_h2_64;
    dp.job[2] = DualJob{1, kPublic4D, kRows2D, 0, d.V, 128, 1.f, 1, 2, g->dv,
                        stride_or(g->dv_stride, d.H * d.V), nullptr, 0.f, nullptr};
    if ((rc = dual(m, dp, 3))) return rc;
  }
  // ================= readout adjoint
  {
    const int per_head = readout_ctas_per_head(d);
    ReadoutBwdParams rp{d.BH, d.H, d.TP, d.NT, d.B, per_head, s.raw, w.dweights, s.lam, w.draw,
                        w.dlam_r, w.dtab_part};
    CUtensorMap m_raw, m_dwt;
    if ((rc = tmap_2d(&m_raw, s.raw, rows, 128, 128))) return rc;
    if ((rc = tmap_2d(&m_dwt, w.dweights, rows, 128, 128))) return rc;
    set_smem(readout_bwd_kernel, kReadoutBwdSmem);
    CYFA_LAUNCH("readout_bwd", st,
                (launch_k(readout_bwd_kernel, d.H * per_head, 256, kReadoutBwdSmem, st, m_tab, m_raw,
                                                                                  m_dwt, rp)));
    if ((rc = launch_status())) return rc;
    cudaStream_t sr = defer_stream(st);  // nothing below reads the table gradient
    CYFA_LAUNCH("dtable_reduce", sr,
                (launch_k(dtable_reduce_kernel, dim3(d.H, 128), 128, 0, sr, w.dtab_part, g->dtable,
                          per_head, g->readout_basis_t, g->dreadout)));
    if ((rc = launch_status())) return rc;
  }
  // ================= pass 1 (queries = q^, keys = k^, values = w)
  {
    ScanParams p{d.BH, d.H, d.TP, d.NT, d.K, 128, kRows2D, kRows2D, s.G, g->dhk, w.h1, g->dhk0,
                 a->scale, nullptr, w.bpart1, a->hk};
    CUtensorMap m_f1, m_ff1;
    if ((rc = tmap_2d(&m_f1, s.s1, uint64_t(d.BH) * d.NT * d.K, 128, 128))) return rc;
    if ((rc = tmap_2d(&m_ff1, s.s1_fin, uint64_t(d.BH) * d.K, 128, 128))) return rc;
    if ((rc = run_scan<true>(d, p, dim3(d.BH, d.K / 128, 2), m_qn, m_draw, m_f1, m_ff1,
                             w.scan_tmp, st)))
      return rc;
    ScoresParams sp{d.BH, d.H, d.TP, d.NT, d.K, 128, kRows2D, kRows2D, s.G, a->scale, w.A,
                    w.Bp};
    CYFA_LAUNCH("tile_scores", st,
                (launch_k(tile_scores_kernel, scores_grid, kScoresThreads, kScoresSmem, st, m_qn,
                          m_kn, m_draw, m_w, sp)));
    if ((rc = launch_status())) return rc;
    DualMaps m;
    DualParams dp{d.BH, d.H, d.TP, d.NT, d.T, s.G};
    // dq^ = B' k^ + scale 2^{G_t} draw S^T ;  dG slots 2.. = q^ . dq^ (per 128 columns)
    m.x1[0] = m_Bp, m.y1[0] = m_kn64, m.x2[0] = m_draw, m.y2[0] = m_s1;
    dp.job[0] = DualJob{0, kRows2D, kRows2D, 1, d.K, 128, a->scale, 0, 3, w.dq1, 0, s.qn, 1.f,
                        w.dG + 2 * slot};
    // dk^ = B'^T q^ + 2^{G_L-G_s} w H^T ;  next K/128 slots = -(k^ . dk^)
    m.x1[1] = m_Bp64, m.y1[1] = m_qn64, m.x2[1] = m_w, m.y2[1] = m_h1;
    dp.job[1] = DualJob{1, kRows2D, kRows2D, 1, d.K, 128, 1.f, 1, 3, w.dk1, 0, s.kn, -1.f,
                        w.dG + (2 + d.K / 128) * slot};
    // dw_b = A^T draw + 2^{G_L-G_s} k^ H  (the write-vector gradient is dw + dw_b)
    m.x1[2] = m_A64, m.y1[2] = m_draw64, m.x2[2] = m_kn, m.y2[2] = m_h1_64;
    dp.job[2] = DualJob{1, kRows2D, kRows2D, 0, 128, d.K, 1.f, 1, 3, w.dw_b, 0, nullptr, 0.f,
                        nullptr};
    if ((rc = dual(m, dp, 3))) return rc;
  }
  // ================= norms, write vector, gates, clock
  int nblk = 0;  // partial rows of the norm-weight gradients
  rc = token_bwd_launch(a->q, a->k, a->q_norm_weight, a->k_norm_weight, s.q_rs, s.k_rs, w.dq1,
                        w.dk1, s.lam, s.beta_h, w.dw, w.dw_b, g->dq, g->dk, w.dqw_part, w.dkw_part,
                        w.dlam_w, w.dbeta_h, d.B, d.T, d.H, d.K,
                        stride_or(a->q_stride, d.H * d.K), stride_or(a->k_stride, d.H * d.K),
                        stride_or(g->dq_stride, d.H * d.K), stride_or(g->dk_stride, d.H * d.K),
                        true, stream, &nblk);
  if (rc) return rc;
  cudaStream_t sc = defer_stream(st);
  CYFA_LAUNCH("column_sum", sc,
              (launch_k(column_sum_kernel, dim3((d.K + 31) / 32, 2), 1024, 0, sc, w.dqw_part,
                        g->dq_norm_weight, nblk, d.K, w.dkw_part, g->dk_norm_weight, 0x7fffffff,
                        nullptr)));
  if ((rc = launch_status())) return rc;
  GatesBwdParams gp{w.dG, ndg, (long long)slot, w.dlam_w, w.dlam_r, w.bpart1, w.bpart2, nsub1,
                    nsub2, w.dbeta_h, g->dclock, g->dg, g->ddelta, g->dbeta, g->dclock0, d.B, d.T,
                    d.H, d.TP, a->lengths};
  CYFA_LAUNCH("gates_bwd", st,
              (launch_k(gates_bwd_kernel, dim3(d.BH, (d.TP + 1023) / 1024), 1024, 0, st, gp)));
  return launch_status();
}

}  // extern "C"
