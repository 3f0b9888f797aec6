/*
 * CyFA B200 hot path -- C ABI.
 *
 * Framework-neutral entry points over raw device pointers and a CUDA stream
 * (passed as void*).  The caller allocates every output and workspace; the
 * library allocates nothing on these paths.  Every entry point checks its
 * arguments on the host before launching and returns a status:
 *   0  ok
 *  >0  argument error (unsupported shape, null or misaligned pointer, ...);
 *      nothing was launched
 *  <0  CUDA launch error (negated cudaError_t)
 * Device-side bounded waits that run out record a code that
 * cyfa_device_error() returns.
 *
 * Layouts (row-major, contiguous):
 *   public  q,k [B,T,H,K] bf16; v [B,T,H,V] bf16; g/delta/beta [B,T,H] f32
 *   head-major (internal, T padded to TP = ceil(T/128)*128):
 *           qn,kn [B,H,TP,K] bf16; w [B,H,TP,128] bf16; G, lam, beta_h [B,H,TP] f32
 *   states  hk [B,H,K,128] f32; hv [B,H,128,V] f32; clock [B,H] f32
 *   table   [H,127,128] f32 (readout R . Phi); table_bf [H,128,128] bf16, row 127 = 0
 *
 * The reference binds these operations as Jittor ops built from generated CUDA
 * strings (cyclic_flow_attention/ops/*); each declaration names the reference
 * interface it replaces.
 */
#ifndef CYFA_H_
#define CYFA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Library version: major*100 + minor. */
int cyfa_version(void);

/* Human-readable text of a status code. */
const char* cyfa_strerror(int status);

/* Reads (and, if reset != 0, clears) the device error word of the current
 * device: 0 = no device-side failure; 1 = a bounded wait timed out.
 * Synchronises the device. */
int cyfa_device_error(int reset);

/* Number of kernels this library has launched in the process (all entry points). */
long long cyfa_launch_count(void);

/* Programmatic dependent launch of the library's kernels: on (1, the default)
 * each kernel may begin while the previous kernel on its stream finishes (it
 * waits on the device before touching memory); off (0) gives plain stream
 * order.  Returns the previous setting. */
int cyfa_set_pdl(int on);

/* State scans with fewer CTAs than SMs (few sequences x heads, long sequences)
 * split their tiles into segments scanned side by side: a pass from zero per
 * segment, the carried states, and the real pass from them.  On (1, the
 * default) or off (0: one serial pass per state slice, the same summation order
 * at every batch size).  Returns the previous setting. */
int cyfa_set_scan_split(int on);

/* Auxiliary stream of the calling thread, or NULL (the default) for none.
 * While set, the entry points called on this thread launch their final
 * parameter-gradient reductions (norm-weight, convolution, gate-parameter and
 * readout-table sums) on it, ordered after the work already issued on the
 * call's stream, so that they overlap the caller's next kernels.  The caller
 * makes its stream wait for the auxiliary stream before reading those
 * gradients or freeing the call's workspace. */
int cyfa_set_aux_stream(void* aux);

/* Turns per-kernel timing on (1) or off (0) and clears earlier records.  While
 * on, every launch is bracketed by CUDA events on its own stream. */
int cyfa_profile_enable(int on);

/* Aggregates the timing records per kernel name: fills up to `max` entries of
 * names / total_ms / counts and returns the number filled (synchronises on the
 * recorded events). */
int cyfa_profile_report(int max, const char** names, float* total_ms, int* counts);

/* ---------------------------------------------------------------- decode
 * One constant-memory decode step (T = 1).
 * Replaces: fused_recurrent_cyfa, cyclic_flow_attention/ops/fused_recurrent.py:10-200
 * (kernel :55-188).
 * q,k [B,1,H,K], v [B,1,H,V] in dtype `dtype` (0 = bf16, 1 = f32); g, delta, beta
 * [B,1,H] f32; table [H,127,128] f32; norm weights [K] f32.  hk_in/hv_in/clock_in
 * may be NULL (zero initial state).  Outputs may alias the inputs (in place).
 * K, V in {128, 256}. */
int cyfa_decode_step(const void* q, const void* k, const void* v, const float* g,
                     const float* delta, const float* beta, const float* table,
                     const float* q_norm_weight, const float* k_norm_weight,
                     const float* hk_in, const float* hv_in, const float* clock_in,
                     float* hk_out, float* hv_out, float* clock_out, void* out, int B, int H,
                     int K, int V, int dtype, float q_eps, float k_eps, float scale,
                     void* stream);

/* One decode step of the CyclicFlowAttention layer between its input and output
 * projections, for all (sequence, head) pairs in one launch (replaces, at T = 1
 * with a cache, reference layers/cyfa.py:299-357 after the q/k/v/g/a/b/d
 * projections and before o_proj: ShortConvolution with a cache :144-181, the gate
 * activations :323-326, fused_recurrent_cyfa, o_norm(o * scale, gate) :350).
 * P: the packed projection rows [B, P_stride] bf16 holding q | k | v (H*K, H*K,
 * H*V columns from column 0) and a | b | d (H columns each from a_col); the conv
 * histories cache_q/k/v [B, W-1, C] bf16 (oldest row first) are shifted in place;
 * wconv_* [C, W] f32; A_log, dt_bias [H] f32, b_bias, d_bias [H] f32 or NULL;
 * gate [B, H*V] bf16 is the output gate's linear without its bias, gate_bias
 * [H*V] bf16, o_norm_weight [V] f32; y [B, H*V] bf16.  State arguments as in
 * cyfa_decode_step (outputs may alias inputs).  K, V in {128, 256}; 2 <= W <= 4. */
typedef struct {
  int B, H, K, V, W;
  int a_col;
  long long P_stride;
  const void* P;
  void* cache_q;
  void* cache_k;
  void* cache_v;
  const float* wconv_q;
  const float* wconv_k;
  const float* wconv_v;
  const float* A_log;
  const float* dt_bias;
  const float* b_bias;
  const float* d_bias;
  const float* table;
  const float* q_norm_weight;
  const float* k_norm_weight;
  const float* hk_in;
  const float* hv_in;
  const float* clock_in;
  float* hk_out;
  float* hv_out;
  float* clock_out;
  const void* gate;
  const void* gate_bias;
  const float* o_norm_weight;
  void* y;
  float q_eps, k_eps, scale, o_eps, o_scale;
} cyfa_decode_layer_args;
int cyfa_decode_layer(const cyfa_decode_layer_args* args, void* stream);

/* fp32 chunk forward (inference): the whole chunk_cyfa forward for fp32 inputs,
 * computed in fp32 throughout as the token recurrence (one CTA per (b, h) runs
 * the decode step over its T tokens), so it equals the reference's generic fp32
 * chunkwise path up to summation order.
 * Replaces: chunk_cyfa with fp32 q/k/v, cyclic_flow_attention/ops/chunk.py:136-161
 * (_scalar_la) and :300-331 (rotation, softmax, table), final state :346-352.
 * q,k [B,T,H,K], v [B,T,H,V], g/delta/beta [B,T,H] f32 contiguous; table
 * [H,127,128] f32; hk0/hv0/clock0 may be NULL (zero state); o [B,T,H,V] f32;
 * hk [B,H,K,128], hv [B,H,128,V], clock [B,H] receive the final state.
 * K, V in {128, 256}.  No gradients: the fp32 training path is not built. */
int cyfa_chunk_fwd_f32(const float* q, const float* k, const float* v, const float* g,
                       const float* delta, const float* beta, const float* table,
                       const float* q_norm_weight, const float* k_norm_weight, const float* hk0,
                       const float* hv0, const float* clock0, float* o, float* hk, float* hv,
                       float* clock, int B, int T, int H, int K, int V, float q_eps, float k_eps,
                       float scale, void* stream);

/* ---------------------------------------------------------------- forward prep
 * Gate layout + clock scan + in-tile log2 gate cumsum.
 * Replaces: head_gates (ops/utils.py:434-492), ClockScan (:229-302),
 * ClockTotal (:305-348), local_log2_cumsum (:495-520); tiles are 128 tokens.
 * clock0 and clock_out may be NULL. */
int cyfa_gates_fwd(const float* g, const float* delta, const float* beta, const float* clock0,
                   float* G, float* lam, float* beta_h, float* clock_out, int B, int T, int H,
                   void* stream);

/* Per-head q/k RMSNorm into head-major bf16 plus the write vector.
 * Replaces: VectorNorm / HeadRMSNorm (ops/qk_norm.py:64-107, 206-239), head_layout
 * (ops/utils.py:351-387), PhaseWriteOnly (ops/utils.py:543-587).  K in {128, 256}. */
int cyfa_token_fwd(const void* q, const void* k, const float* q_norm_weight,
                   const float* k_norm_weight, const float* lam, const float* beta_h, void* qn,
                   void* kn, void* w, float* q_rs, float* k_rs, int B, int T, int H, int K,
                   float q_eps, float k_eps, void* stream);

/* ---------------------------------------------------------------- backward prep
 * Adjoint of cyfa_token_fwd.  dqn/dkn [B,H,TP,K] f32, dw [B,H,TP,128] f32 in;
 * dq/dk public-layout bf16, norm-weight partial sums
 * [min(ceil(B*H*TP/8), 444), K] f32 (sum the rows for the weight gradient),
 * dlam (write-vector part) and dbeta_h [B,H,TP] f32 out.
 * Replaces: VectorNorm.grad (ops/qk_norm.py:109-165), PhaseWriteOnly.grad
 * (ops/utils.py:589-640). */
int cyfa_token_bwd(const void* q, const void* k, const float* q_norm_weight,
                   const float* k_norm_weight, const float* q_rs, const float* k_rs,
                   const float* dqn, const float* dkn, const float* lam, const float* beta_h,
                   const float* dw, void* dq, void* dk, float* dqw_part, float* dkw_part,
                   float* dlam, float* dbeta_h, int B, int T, int H, int K, void* stream);

/* Adjoint of cyfa_gates_fwd: dG, dlam, dbeta_h [B,H,TP] (+ dclock [B,H] or NULL)
 * -> dg, ddelta, dbeta [B,T,H] and dclock0 [B,H] (or NULL).  dG is the gradient
 * w.r.t. the natural-log in-tile gate cumsum (G / log2(e)).
 * Replaces: ClockScan.grad (ops/utils.py:297-298), ClockTotal.grad (:343-344),
 * HeadGates.grad (:459-488) and the local cumsum adjoint. */
int cyfa_gates_bwd(const float* dG, const float* dlam, const float* dbeta_h,
                   const float* dclock, float* dg, float* ddelta, float* dbeta,
                   float* dclock0, int B, int T, int H, void* stream);

/* ---------------------------------------------------------------- chunk op
 * Chunked CyFA (both ScalarGatedLA passes joined by the softmax slot readout).
 * Replaces: chunk_cyfa, cyclic_flow_attention/ops/chunk.py:164-353, with its fused
 * internals first_readout (ops/chunk_readout.py:961-991,1124-1136), scalar_la /
 * ScalarAttention (ops/chunk.py:30-79), state_forward (ops/chunk_h.py:338) and
 * output_forward (ops/chunk_o.py:394-613).  K in {128, 256}, V in {128, 256},
 * 128 slot rows.  The caller owns `saved` (cyfa_chunk_saved_bytes) and keeps it
 * for cyfa_chunk_bwd; the final state outputs are always written because the
 * backward pass reads them.  q, k and v may be column slices of wider rows (a
 * packed projection output): their token strides are given in elements (multiples
 * of 8, >= the row width; 0 = dense). */
typedef struct {
  int B, T, H, K, V;
  float q_eps, k_eps, scale;
  const void* q;                /* [B,T,H,K] bf16 */
  const void* k;                /* [B,T,H,K] bf16 */
  const void* v;                /* [B,T,H,V] bf16 */
  const float* g;               /* [B,T,H] log decay (<= 0) */
  const float* delta;           /* [B,T,H] clock increment */
  const float* beta;            /* [B,T,H] write strength */
  const float* q_norm_weight;   /* [K] */
  const float* k_norm_weight;   /* [K] */
  const void* table_bf;         /* [H,128,128] bf16 readout table, row 127 zero */
  const float* hk0;             /* [B,H,K,128] or NULL */
  const float* hv0;             /* [B,H,128,V] or NULL */
  const float* clock0;          /* [B,H] or NULL */
  void* o;                      /* out [B,T,H,V] bf16 */
  float* hk;                    /* out [B,H,K,128] final key state */
  float* hv;                    /* out [B,H,128,V] final value state */
  float* clock;                 /* out [B,H] final clock */
  long long q_stride;           /* elements between consecutive tokens of q (0 = H*K) */
  long long k_stride;           /* ... of k (0 = H*K) */
  long long v_stride;           /* ... of v (0 = H*V) */
  const int* lengths;           /* [B] valid tokens of each sequence, or NULL (all T): the
                                   tokens past it are right padding, neutral for the
                                   states and the clock (g = delta = beta = 0 there, as
                                   the reference layer masks them, layers/cyfa.py:304-308,
                                   326-328); their gate gradients are zero */
} cyfa_chunk_fwd_args;

size_t cyfa_chunk_saved_bytes(int B, int T, int H, int K, int V);

int cyfa_chunk_fwd(const cyfa_chunk_fwd_args* args, void* saved, size_t saved_bytes,
                   void* stream);

/* Backward of cyfa_chunk_fwd.  `fwd` repeats the forward arguments (its o may be
 * NULL; hk, hv and clock must hold the forward's final state).  d_o [B,T,H,V] bf16
 * is required; dhk, dhv, dclock (gradients of the final state) may be NULL.
 * Outputs: dq, dk [B,T,H,K] bf16, dv [B,T,H,V] bf16, dg, ddelta, dbeta [B,T,H] f32,
 * dtable [H,128,128] f32 (gradient of the readout table R.Phi; row 127 unused),
 * dq_norm_weight, dk_norm_weight [K] f32, and dhk0, dhv0, dclock0 (initial-state
 * gradients, each may be NULL).  `work` is scratch (cyfa_chunk_work_bytes).
 * Replaces: ScalarAttention.grad / scalar_grad (ops/chunk.py:51-71,
 * ops/chunk_bwd.py:1015-1041), FirstReadoutCompact.grad / readout_grad_compact
 * (ops/chunk_readout.py:976-987,401-621), state_backward (ops/chunk_h.py:342),
 * PhaseWriteOnly.grad, ClockScan.grad, HeadGates.grad (ops/utils.py) and
 * VectorNorm.grad (ops/qk_norm.py:109-165). */
typedef struct {
  cyfa_chunk_fwd_args fwd;
  const void* d_o;              /* [B,T,H,V] bf16 */
  const float* dhk;             /* [B,H,K,128] or NULL */
  const float* dhv;             /* [B,H,128,V] or NULL */
  const float* dclock;          /* [B,H] or NULL */
  void* dq;                     /* out [B,T,H,K] bf16 */
  void* dk;                     /* out [B,T,H,K] bf16 */
  void* dv;                     /* out [B,T,H,V] bf16 */
  float* dg;                    /* out [B,T,H] */
  float* ddelta;                /* out [B,T,H] */
  float* dbeta;                 /* out [B,T,H] */
  float* dtable;                /* out [H,128,128] */
  float* dq_norm_weight;        /* out [K] */
  float* dk_norm_weight;        /* out [K] */
  float* dhk0;                  /* out [B,H,K,128] or NULL */
  float* dhv0;                  /* out [B,H,128,V] or NULL */
  float* dclock0;               /* out [B,H] or NULL */
  long long dq_stride;          /* token stride of dq (0 = H*K) */
  long long dk_stride;          /* token stride of dk (0 = H*K) */
  long long dv_stride;          /* token stride of dv (0 = H*V) */
  const float* readout_basis_t; /* Phi^T [128,127] f32, or NULL */
  float* dreadout;              /* out [H,127,127], or NULL: the readout gradient
                                   (cyfa_readout_table_grad of dtable) in the same
                                   launch as dtable */
} cyfa_chunk_bwd_args;

/* Readout table in the kernels' layout (replaces the table product of
 * cyclic_flow_attention/ops/chunk.py:281, jt.matmul(readout, _basis(M))):
 * table_bf[h][r][m] = bf16(sum_k readout[h][r][k] basis[k][m]) for r < 127, row
 * 127 zero.  readout [H,127,127] f32, basis (the real Fourier basis Phi)
 * [127,128] f32, table_bf [H,128,128] bf16. */
int cyfa_readout_table(const float* readout, const float* basis, void* table_bf, int H,
                       void* stream);

/* Adjoint of cyfa_readout_table: dreadout[h][r][k] = sum_m dtable[h][r][m]
 * basis[k][m] for r, k < 127.  dtable [H,128,128] f32 (as cyfa_chunk_bwd writes
 * it), basis_t = Phi^T [128,127] f32, dreadout [H,127,127] f32. */
int cyfa_readout_table_grad(const float* dtable, const float* basis_t, float* dreadout, int H,
                            void* stream);

size_t cyfa_chunk_work_bytes(int B, int T, int H, int K, int V);

int cyfa_chunk_bwd(const cyfa_chunk_bwd_args* args, const void* saved, size_t saved_bytes,
                   void* work, size_t work_bytes, void* stream);

/* ---------------------------------------------------------------- layer glue
 * Causal depthwise short convolution without activation.
 * Replaces: ShortConvolution (cyclic_flow_attention/layers/cyfa.py:138-233).
 * x [B,T,C] bf16 with token stride x_stride (elements); cache [B,W-1,C] bf16 (the
 * history before t = 0) or NULL for zeros; w [C,W] f32; bias [C] f32 or NULL;
 * y [B,T,C] bf16 dense.  C % 8 == 0, 1 <= W <= 4. */
int cyfa_short_conv_fwd(const void* x, long long x_stride, const void* cache, const float* w,
                        const float* bias, void* y, int B, int T, int C, int W, void* stream);

size_t cyfa_short_conv_work_bytes(int B, int T, int C, int W);

/* Adjoint of cyfa_short_conv_fwd without cache: dy [B,T,C] bf16 dense -> dx (token
 * stride dx_stride), dw [C,W] f32 and dbias [C] f32 (or NULL). */
int cyfa_short_conv_bwd(const void* x, long long x_stride, const float* w, const void* dy,
                        void* dx, long long dx_stride, float* dw, float* dbias, int B, int T,
                        int C, int W, void* work, size_t work_bytes, void* stream);

/* Gate activations of the layer: g = -exp(A_log) softplus(a + dt_bias),
 * delta = sigmoid(d + d_bias), beta = sigmoid(b + b_bias), all [rows, H] f32 out;
 * a, b, d are bf16 projection outputs with token strides; the biases [H] f32 may
 * be NULL.  Replaces layers/cyfa.py:323-326. */
int cyfa_gate_act_fwd(const void* a, long long a_stride, const void* b, long long b_stride,
                      const void* d, long long d_stride, const float* A_log,
                      const float* dt_bias, const float* b_bias, const float* d_bias, float* g,
                      float* delta, float* beta, int rows, int H, void* stream);

size_t cyfa_gate_act_work_bytes(int rows, int H);

/* Adjoint of cyfa_gate_act_fwd: da, db, dd bf16 (token strides), and the
 * parameter gradients dA_log, ddt_bias, db_bias, dd_bias [H] (the last two may be
 * NULL). */
int cyfa_gate_act_bwd(const void* a, long long a_stride, const void* b, long long b_stride,
                      const void* d, long long d_stride, const float* A_log,
                      const float* dt_bias, const float* b_bias, const float* d_bias,
                      const float* dg, const float* ddelta, const float* dbeta, void* da,
                      long long da_stride, void* db, long long db_stride, void* dd,
                      long long dd_stride, float* dA_log, float* ddt_bias, float* db_bias,
                      float* dd_bias, int rows, int H, void* work, size_t work_bytes,
                      void* stream);

/* Gated output norm: y = RMSNorm(scale * x) * w * sigmoid(gate) over rows of D
 * (x, gate, y [rows, D] bf16; rstd [rows] f32 saved for the backward).
 * Replaces: o_norm(o * (num_slots - 1), gate) (layers/cyfa.py:350, RMSNorm :62-135). */
int cyfa_gated_norm_fwd(const void* x, const void* gate, const float* w, float eps, float scale,
                        void* y, float* rstd, int rows, int D, void* stream);

size_t cyfa_gated_norm_work_bytes(int rows, int D);

int cyfa_gated_norm_bwd(const void* x, const void* gate, const float* w, float scale,
                        const float* rstd, const void* dy, void* dx, void* dgate, float* dw,
                        int rows, int D, void* work, size_t work_bytes, void* stream);

/* Gated norm with the output gate's bias folded in: sigmoid(gate + b[head])
 * where rows are (token, head) pairs, head = row % H, b [H*D] bf16 (the bias of
 * the gate's second linear, reference layers/cyfa.py:292-295,349-350).  The
 * backward also returns dgate_bias [H*D] f32 (fixed-order sums).  Work buffer:
 * cyfa_gated_norm_bias_work_bytes(rows, D, H). */
int cyfa_gated_norm_bias_fwd(const void* x, const void* gate, const void* gate_bias, int H,
                             const float* w, float eps, float scale, void* y, float* rstd,
                             int rows, int D, void* stream);
size_t cyfa_gated_norm_bias_work_bytes(int rows, int D, int H);
int cyfa_gated_norm_bias_bwd(const void* x, const void* gate, const void* gate_bias, int H,
                             const float* w, float scale, const float* rstd, const void* dy,
                             void* dx, void* dgate, float* dw, float* dgate_bias, int rows, int D,
                             void* work, size_t work_bytes, void* stream);

/* The output gate's second linear fused into the biased gated norm (replaces the
 * g_proj second linear plus o_norm of reference layers/cyfa.py:292-295,349-350):
 *   gate = bf16(gin Wg^T),  y = RMSNorm(scale * x) * w * sigmoid(gate + gate_bias)
 * x, y: [tokens, H, D] bf16 (D = 128 or 256); gin: [tokens, Kg] bf16 rows
 * gin_stride elements apart (Kg a multiple of 64; a column view of a packed
 * projection is fine); gate_w: [H*D, Kg] bf16 row-major; gate_bias: [H*D] bf16 or
 * NULL; rstd: [tokens*H] f32.  gate_out ([tokens, H*D] bf16, the gate before its
 * bias, as cyfa_gated_norm_bias_bwd reads it) is written when not NULL.  The
 * linear accumulates in fp32 on the tensor cores and is rounded to bf16 before
 * the bias, as a bf16 linear's output is. */
int cyfa_gated_norm_gate_fwd(const void* x, const void* gin, long long gin_stride,
                             const void* gate_w, const void* gate_bias, int H, int Kg,
                             const float* w, float eps, float scale, void* y, float* rstd,
                             void* gate_out, int tokens, int D, void* stream);

/* Allocation-free variant of cyfa_gated_norm_bwd, for callers that cannot hand the
 * library a workspace: bindings whose signature carries only the op's tensors, or
 * processes whose device memory belongs entirely to a framework allocator.  No
 * counterpart in the reference.  The weight-gradient partials live in a fixed
 * device array inside the library (296 KiB, held on every GPU that loads the
 * library until exit) instead of a caller buffer; D in {128, 256}, any rows.
 * The first call on each device looks up that array's device address
 * (cudaGetSymbolAddress); make the first call before any stream capture.  All
 * calls share the array: each call overwrites what it reads, but calls whose
 * kernels overlap on the GPU race.  The looked-up address is kept for the life of
 * the process: do not call it again on a device after cudaDeviceReset (or any
 * other reset of that device's primary context).  Calls no allocator. */
int cyfa_gated_norm_bwd_static(const void* x, const void* gate, const float* w, float scale,
                               const float* rstd, const void* dy, void* dx, void* dgate,
                               float* dw, int rows, int D, void* stream);

/* ---------------------------------------------------------------- LM decode glue
 * One launch each for the glue of a recurrent decode step of the CyFA language
 * model (batch x hidden rows per step, so launch count is what they save).
 *
 * Residual add + RMSNorm of the decoder blocks.  Replaces: residual = x + y and
 * RMSNorm (models/cyfa/modeling_cyfa.py:52-55,64-69; RMSNorm layers/cyfa.py:62-135).
 * If y != NULL, x = bf16(x + y) in place first; then out = bf16(x * rsqrt(mean(x^2)
 * + eps) * w).  x, y, out [rows, D] bf16, w [D] f32; D % 8 == 0, D <= 8192, all
 * 16-byte aligned. */
int cyfa_add_rmsnorm(void* x, const void* y, const float* w, float eps, void* out, int rows,
                     int D, void* stream);

/* The q, k and v short convolutions of one decode token.  Replaces:
 * ShortConvolution.execute with a cache at T = 1 (layers/cyfa.py:144-181), three
 * convolutions in one launch.  Row b of x holds the pre-convolution q|k|v values
 * (widths Cq, Ck, Cv) at x + b * x_stride; the caches [B, W-1, C] bf16 (oldest row
 * first) are shifted in place to end with this token; w [C, W] f32; y [B, C] bf16.
 * 2 <= W <= 4, widths and x_stride multiples of 8, all pointers 16-byte aligned, no
 * bias. */
int cyfa_decode_conv(const void* x, long long x_stride, void* cache_q, void* cache_k,
                     void* cache_v, const float* wq, const float* wk, const float* wv, void* yq,
                     void* yk, void* yv, int B, int Cq, int Ck, int Cv, int W, void* stream);

/* Gated MLP activation: out = bf16(g sigmoid(g) u) in fp32, gu [rows, 2 * mid] bf16
 * (gate columns first, then up columns), out [rows, mid] bf16; mid % 8 == 0.
 * Replaces: GatedMLP.execute (models/cyfa/modeling_cyfa.py:22-27). */
int cyfa_swiglu(const void* gu, void* out, int rows, int mid, void* stream);

/* ---------------------------------------------------------------- self test
 * C[128,N] = A * B through TMA + tcgen05 (test hook for the UMMA descriptor and
 * swizzle encodings).  A is [128,K] (a_mn = 0) or [K,128] (a_mn = 1); B is [N,K]
 * (b_mn = 0) or [K,N] (b_mn = 1); bf16, row-major.  K in {64,...,256} step 64,
 * N in {64,128,256}.  No counterpart in the reference. */
int cyfa_selftest_umma(const void* a, const void* b, float* c, int K, int N, int a_mn,
                       int b_mn, void* stream);

/* ---------------------------------------------------------------- gradient buckets
 * Data-parallel plumbing: the weight gradients of a bucket are gathered into one
 * flat fp32 buffer for the all-reduce and the averaged values are written back.
 * The reference flattens its fp32 gradient bucket with Jittor ops before the MPI
 * all-reduce (training/optim.py:52-63); these replace those copies with one
 * launch per bucket each way. */
typedef struct {
  void* ptr;          /* the tensor's contiguous data, 16-byte aligned */
  long long n;        /* elements */
  long long offset;   /* first element in the flat bucket, a multiple of 8 */
  int dtype;          /* 0 = f32, 1 = bf16 */
} cyfa_bucket_piece;

/* flat[offset + i] = float(ptr[i]) for every piece (one launch per 64 pieces). */
int cyfa_bucket_gather(const cyfa_bucket_piece* pieces, int count, float* flat, void* stream);

/* ptr[i] = dtype(scale * flat[offset + i]) for every piece (one launch per 64 pieces). */
int cyfa_bucket_scatter(const cyfa_bucket_piece* pieces, int count, const float* flat,
                        float scale, void* stream);

/* ---------------------------------------------------------------- optimizer
 * AdamW with fp32 master weights and moments.  Replaces: AdamW.step,
 * training/optim.py:96-124.  The masters, moments and the (all-reduced,
 * accumulated) gradient live in flat fp32 buffers; `params` lists each
 * parameter tensor (bf16 or f32) with its element offset into those buffers
 * (a multiple of 8; every pointer 16-byte aligned).  One launch per 64
 * parameters updates m, v and the master in the reference's formula order and
 * writes the master rounded to the parameter's dtype; `step` >= 1 is the
 * update count used for the bias corrections. */
int cyfa_adamw_step(const cyfa_bucket_piece* params, int count, float* master, float* m, float* v,
                    const float* grad, float lr, float beta1, float beta2, float eps,
                    float weight_decay, int step, void* stream);

/* Gradient clipping by the global L2 norm.  Replaces: AdamW.clip_grad_norm,
 * training/optim.py:74-89.  grad [n] f32 is scaled in place by
 * min(max_norm / (norm + 1e-6), 1); the norm is written to norm_out (device
 * f32, may be NULL).  Sums run in a fixed order (deterministic).  work:
 * cyfa_grad_clip_work_bytes() bytes of device memory. */
size_t cyfa_grad_clip_work_bytes(void);
int cyfa_grad_clip(float* grad, long long n, float max_norm, float* norm_out, void* work,
                   size_t work_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CYFA_H_ */
