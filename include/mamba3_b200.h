/*
 * mamba3_b200.h -- C ABI of the B200 (sm_100a) Mamba-3 scan library (libmamba3_b200.so).
 *
 * Every entry point takes plain device pointers wrapped in m3_tensor descriptors (shape +
 * element strides), launches on the caller's CUDA stream and returns an m3_status; the
 * text of the last error on the calling thread is available from m3_last_error_string().
 * Nothing here allocates device memory: the caller owns every input, output and
 * workspace buffer. Host (CPU) pointers are rejected; there is no CPU fallback.
 *
 * Reference interfaces replaced (upstream Aiyoniganmaaiya/mamba3-ssm v0.2.1):
 *   - the pybind functions siso_scan / mimo_state built by load_inline
 *     (mamba3_ssm/cuda_backend.py:319-356) and their raw launchers
 *     (cuda_backend.py:236-301), reached from ssm_scan_siso / ssm_scan_mimo
 *     (mamba3_ssm/ops.py:126-242);
 *   - the per-token recurrence written in PyTorch inside Mamba3.step
 *     (mamba3_ssm/layer.py:296-371), which has no native boundary upstream.
 *
 * Layout conventions (reference layouts, innermost dimension contiguous):
 *   x, y, dx, dy     (B, L, H, P)        f32 / bf16 / f16
 *   SISO B, C        (B, L, H, D)        f32 / bf16 / f16
 *   MIMO B, C        (B, L, R, H, D)     f32 / bf16 / f16
 *   ADT, DT, trap    (B, L, H)           f32, any strides (trap is a logit: the kernels
 *                                        apply the sigmoid, as ops.py:148 does)
 *   D                (H)                 f32
 *   mimo_x, mimo_o   (H, R, P)           f32 / bf16
 *   SISO states      (B, H, P, D)        f32 contiguous
 *   MIMO states      (B, H, D)           f32 contiguous
 */
#ifndef MAMBA3_B200_H
#define MAMBA3_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define M3_ABI_VERSION 1
#define M3_MAX_DIMS 6

typedef enum m3_dtype {
  M3_FLOAT32 = 0,
  M3_BFLOAT16 = 1,
  M3_FLOAT16 = 2,
  M3_INT64 = 3 /* token ids (m3_argmax_rows) */
} m3_dtype;

typedef enum m3_status {
  M3_OK = 0,
  M3_ERR_INVALID_ARGUMENT = 1, /* shape, stride, dtype or pointer problem            */
  M3_ERR_UNSUPPORTED = 2,      /* valid request outside the compiled kernel variants  */
  M3_ERR_CUDA = 3,             /* a CUDA runtime call or kernel launch failed         */
  M3_ERR_WORKSPACE = 4         /* workspace missing or too small                      */
} m3_status;

/* A strided view of device memory. data == NULL marks an absent optional argument. */
typedef struct m3_tensor {
  void* data;
  int32_t dtype; /* m3_dtype */
  int32_t ndim;
  int64_t shape[M3_MAX_DIMS];
  int64_t stride[M3_MAX_DIMS]; /* in elements */
} m3_tensor;

/* Dimensions of one Mamba3 mixer (mamba3_ssm/layer.py:82-115). */
typedef struct m3_layer_dims {
  int32_t d_model;
  int32_t d_inner;         /* expand * d_model                                */
  int32_t nheads;          /* H = d_inner / headdim                            */
  int32_t headdim;         /* P                                                */
  int32_t d_state;         /* D                                                */
  int32_t ngroups;         /* G (B/C groups broadcast to heads)                */
  int32_t mimo_rank;       /* R (1 for SISO)                                   */
  int32_t num_rope_angles; /* S = split / 2                                    */
  int32_t rope_split;      /* leading state dims that rotate (even)            */
  float A_floor;           /* layer.py:207                                     */
  float norm_eps;          /* RMSNorm eps of B_norm / C_norm (ops.py:97)       */
} m3_layer_dims;

/* ---------------------------------------------------------------------------------
 * Library information
 * ------------------------------------------------------------------------------- */
int m3_abi_version(void);
const char* m3_last_error_string(void);

/* ---------------------------------------------------------------------------------
 * SISO scan, forward.  Replaces siso_scan(x, B, C, decay, dt, tr, D)
 * (cuda_backend.py:319-336 -> siso_scan_launcher :236-267 -> siso_scan_kernel :35-111)
 * as called by ssm_scan_siso (ops.py:126-177); unlike the reference it takes ADT and
 * the trap logit and applies exp / sigmoid itself (ops.py:146-148).
 *   y[b,t,h,:] = h_t C_t + D[h] x_t,  h_t = e^{ADT} h_{t-1} + DT*blend(x_t B_t, x_{t-1}B_{t-1})
 * h0, bx0      optional initial state / previous B*x (B,H,P,D) f32; absent = zeros.
 * h_last, bx_last  optional outputs (B,H,P,D) f32: state and B*x after the last step
 *              (the decode-cache pair of layer.py:284-285).
 * ------------------------------------------------------------------------------- */
int m3_siso_scan_fwd(const m3_tensor* x, const m3_tensor* B, const m3_tensor* C,
                     const m3_tensor* ADT, const m3_tensor* DT, const m3_tensor* trap,
                     const m3_tensor* D, const m3_tensor* h0, const m3_tensor* bx0,
                     m3_tensor* y, m3_tensor* h_last, m3_tensor* bx_last, void* stream);

/* SISO scan, backward. The reference has no backward kernel (its CUDA tier drops the
 * gradient; cuda_backend.py:327); this returns the gradients autograd produces through
 * the loop of ops.py:166-175.
 * workspace: buffer of at least m3_siso_scan_bwd_workspace_size() bytes, 256-byte
 * aligned. For bf16 inputs with headdim 64 and d_state 128 or 64 a workspace of that size lets
 * the call take the chunked tensor-core path (it recomputes the forward's chunk states
 * into the workspace first); a workspace of only 4 * batch * nheads * seqlen bytes selects
 * the CUDA-core path, which every shape supports.
 * dD (H) f32 is overwritten. dh0 / dbx0 optional (B,H,P,D) f32 outputs. */
size_t m3_siso_scan_bwd_workspace_size(int64_t batch, int64_t seqlen, int64_t nheads,
                                       int64_t headdim, int64_t dstate);
int m3_siso_scan_bwd(const m3_tensor* x, const m3_tensor* B, const m3_tensor* C,
                     const m3_tensor* ADT, const m3_tensor* DT, const m3_tensor* trap,
                     const m3_tensor* D, const m3_tensor* h0, const m3_tensor* bx0,
                     const m3_tensor* dy, m3_tensor* dx, m3_tensor* dB, m3_tensor* dC,
                     m3_tensor* dADT, m3_tensor* dDT, m3_tensor* dtrap, m3_tensor* dD,
                     m3_tensor* dh0, m3_tensor* dbx0, void* workspace,
                     size_t workspace_bytes, void* stream);

/* SISO scan, backward, without any device allocation by the caller or the library.
 * No counterpart in the reference. Same arguments and results as m3_siso_scan_bwd, minus
 * the workspace: the per-position workspace lives in a fixed device array inside this
 * library (M3_NOALLOC_MAX_POSITIONS floats = 8 MiB, held by every GPU that loads the
 * library until the process exits). For callers that may not allocate device memory at the
 * point of the backward call, e.g. a host framework that owns a fixed device-memory budget
 * and forbids side allocations by extensions.
 *   - batch * seqlen * nheads above M3_NOALLOC_MAX_POSITIONS returns M3_ERR_WORKSPACE.
 *   - The first call on a device looks up the array's device address (once per device,
 *     with that device current); make that first call before any stream capture.
 *   - Every call on a GPU shares the one array: calls whose kernels overlap on that GPU
 *     (different streams, or host threads) race and produce wrong gradients. Serialise them.
 *   - Nothing carries over between calls: each call writes every scratch entry it reads.
 *   - Which backward runs depends on the size, because the array is the whole workspace:
 *     for bf16 inputs with headdim 64 and d_state 128 or 64 the tensor-core backward runs
 *     while its chunk states plus scratch fit, i.e. while
 *       (16384 * chunks rounded up to 256) + 12 * positions + 16 * chunks,
 *       chunks = batch * nheads * ceil(seqlen / 128),
 *     is at most 8 MiB (about 59K positions); above that, and for every other shape, the
 *     CUDA-core backward runs (several times slower at those sizes, and it rounds bf16
 *     gradients differently, within the same bf16 tolerance). */
#define M3_NOALLOC_MAX_POSITIONS (2 * 1024 * 1024)
int m3_siso_scan_bwd_noalloc(const m3_tensor* x, const m3_tensor* B, const m3_tensor* C,
                             const m3_tensor* ADT, const m3_tensor* DT, const m3_tensor* trap,
                             const m3_tensor* D, const m3_tensor* h0, const m3_tensor* bx0,
                             const m3_tensor* dy, m3_tensor* dx, m3_tensor* dB, m3_tensor* dC,
                             m3_tensor* dADT, m3_tensor* dDT, m3_tensor* dtrap, m3_tensor* dD,
                             m3_tensor* dh0, m3_tensor* dbx0, void* stream);

/* SISO scan with saved chunk states (no counterpart in the reference; replaces the pair
 * ssm_scan_siso forward / autograd backward of ops.py:145-181 when the forward is run for
 * training). The forward additionally writes the carried state at the start of every
 * 128-step chunk (bf16, m3_siso_scan_kstates_size bytes, 256-byte aligned); the backward
 * reads them instead of recomputing the forward.
 *   m3_siso_scan_kstates_size  bytes of the state array; 0 when the chunked kernels do not
 *                              cover the request (then use m3_siso_scan_fwd / _bwd).
 *                              x_dtype / bc_dtype are m3_dtype codes.
 *   m3_siso_scan_fwd_kstates   as m3_siso_scan_fwd, plus the state array (output).
 *   m3_siso_scan_bwd_kstates   as m3_siso_scan_bwd, with the state array of the forward on
 *                              the same inputs and a workspace of
 *                              m3_siso_scan_bwd_kstates_workspace_size bytes.
 * M3_ERR_UNSUPPORTED when the inputs are outside the chunked kernels (dtype, headdim 64,
 * d_state 128 or 64, 16-byte aligned rows). The state array holds 128 rows per chunk
 * for either d_state. */
size_t m3_siso_scan_kstates_size(int64_t batch, int64_t seqlen, int64_t nheads, int64_t headdim,
                                 int64_t dstate, int x_dtype, int bc_dtype);
size_t m3_siso_scan_bwd_kstates_workspace_size(int64_t batch, int64_t seqlen, int64_t nheads);
int m3_siso_scan_fwd_kstates(const m3_tensor* x, const m3_tensor* B, const m3_tensor* C,
                             const m3_tensor* ADT, const m3_tensor* DT, const m3_tensor* trap,
                             const m3_tensor* D, const m3_tensor* h0, const m3_tensor* bx0,
                             m3_tensor* y, m3_tensor* h_last, m3_tensor* bx_last,
                             void* kstates, size_t kstates_bytes, void* stream);
int m3_siso_scan_bwd_kstates(const m3_tensor* x, const m3_tensor* B, const m3_tensor* C,
                             const m3_tensor* ADT, const m3_tensor* DT, const m3_tensor* trap,
                             const m3_tensor* D, const m3_tensor* h0, const m3_tensor* bx0,
                             const m3_tensor* dy, m3_tensor* dx, m3_tensor* dB, m3_tensor* dC,
                             m3_tensor* dADT, m3_tensor* dDT, m3_tensor* dtrap, m3_tensor* dD,
                             m3_tensor* dh0, m3_tensor* dbx0, const void* kstates,
                             size_t kstates_bytes, void* workspace, size_t workspace_bytes,
                             void* stream);

/* ---------------------------------------------------------------------------------
 * MIMO scan, forward.  Replaces mimo_state_cuda (cuda_backend.py:419-463: einsum ->
 * mimo_state(x_mixed, ...) :339-356 -> mimo_state_kernel :123-204 -> einsum) as called
 * by ssm_scan_mimo (ops.py:184-242). The rank-R projections through mimo_x / mimo_o
 * and the D skip are fused into the same kernel.
 * ------------------------------------------------------------------------------- */
int m3_mimo_scan_fwd(const m3_tensor* x, const m3_tensor* B, const m3_tensor* C,
                     const m3_tensor* ADT, const m3_tensor* DT, const m3_tensor* trap,
                     const m3_tensor* D, const m3_tensor* mimo_x, const m3_tensor* mimo_o,
                     const m3_tensor* h0, const m3_tensor* bx0, m3_tensor* y,
                     m3_tensor* h_last, m3_tensor* bx_last, void* stream);

/* MIMO scan, backward (gradients of ops.py:226-240). dD, dmimo_x, dmimo_o are f32 and
 * overwritten. */
/* Chunk-parallel MIMO forward: same operands and results as m3_mimo_scan_fwd, plus a
 * caller-provided device workspace (16-byte aligned) of at least
 * m3_mimo_scan_fwd_workspace_size(...) bytes (about 8 * batch * nheads * ceil(seqlen / 16)
 * * (dstate + 1) bytes: per (b, h, chunk) the published states and decay with their status
 * words). The time axis is cut into 16 / 32 / 64-step chunks; one pass reads x, B and C
 * once (TMA boxes), each chunk finding the state that enters it by looking back over the
 * chunks before it. Inputs whose rows the TMA cannot describe (x / B / C not 16-byte
 * aligned or with strides that are not whole 16-byte units) take a three-pass form (local
 * states, carry pass, outputs). Replaces the same reference path as m3_mimo_scan_fwd
 * (cuda_backend.py:419-463, ops.py:226-240). */
size_t m3_mimo_scan_fwd_workspace_size(int64_t batch, int64_t seqlen, int64_t nheads, int64_t dstate);
int m3_mimo_scan_fwd_ws(const m3_tensor* x, const m3_tensor* B, const m3_tensor* C, const m3_tensor* ADT,
                        const m3_tensor* DT, const m3_tensor* trap, const m3_tensor* D,
                        const m3_tensor* mimo_x, const m3_tensor* mimo_o, const m3_tensor* h0,
                        const m3_tensor* bx0, m3_tensor* y, m3_tensor* h_last, m3_tensor* bx_last,
                        void* workspace, size_t workspace_bytes, void* stream);

size_t m3_mimo_scan_bwd_workspace_size(int64_t batch, int64_t seqlen, int64_t nheads,
                                       int64_t headdim, int64_t dstate, int64_t rank);
int m3_mimo_scan_bwd(const m3_tensor* x, const m3_tensor* B, const m3_tensor* C,
                     const m3_tensor* ADT, const m3_tensor* DT, const m3_tensor* trap,
                     const m3_tensor* D, const m3_tensor* mimo_x, const m3_tensor* mimo_o,
                     const m3_tensor* h0, const m3_tensor* bx0, const m3_tensor* dy,
                     m3_tensor* dx, m3_tensor* dB, m3_tensor* dC, m3_tensor* dADT,
                     m3_tensor* dDT, m3_tensor* dtrap, m3_tensor* dD, m3_tensor* dmimo_x,
                     m3_tensor* dmimo_o, m3_tensor* dh0, m3_tensor* dbx0, void* workspace,
                     size_t workspace_bytes, void* stream);

/* MIMO backward from the forward's workspace: same operands and results as
 * m3_mimo_scan_bwd, plus the device workspace a preceding m3_mimo_scan_fwd_ws call filled
 * with the same inputs (x, B, C, ADT, DT, trap, D, mimo_x, h0, bx0). Where that forward ran
 * its single-pass kernel, the backward is one pass too: it reads the forward's published
 * chunk-end states instead of recomputing the forward, finds each chunk's adjoint carry by
 * looking ahead over the chunks after it, and reads x, B, C and dy once (TMA boxes).
 * Otherwise (inputs the TMA cannot describe, fwd_workspace NULL or too small) it runs the
 * m3_mimo_scan_bwd kernels. workspace: at least m3_mimo_scan_bwd_ws_workspace_size(...)
 * bytes, 16-byte aligned. Same reference path as m3_mimo_scan_bwd (the gradients of
 * ops.py:226-240). */
size_t m3_mimo_scan_bwd_ws_workspace_size(int64_t batch, int64_t seqlen, int64_t nheads,
                                          int64_t headdim, int64_t dstate, int64_t rank);
int m3_mimo_scan_bwd_ws(const m3_tensor* x, const m3_tensor* B, const m3_tensor* C,
                        const m3_tensor* ADT, const m3_tensor* DT, const m3_tensor* trap,
                        const m3_tensor* D, const m3_tensor* mimo_x, const m3_tensor* mimo_o,
                        const m3_tensor* h0, const m3_tensor* bx0, const m3_tensor* dy,
                        m3_tensor* dx, m3_tensor* dB, m3_tensor* dC, m3_tensor* dADT,
                        m3_tensor* dDT, m3_tensor* dtrap, m3_tensor* dD, m3_tensor* dmimo_x,
                        m3_tensor* dmimo_o, m3_tensor* dh0, m3_tensor* dbx0,
                        const void* fwd_workspace, size_t fwd_workspace_bytes, void* workspace,
                        size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------------
 * Single-token decode step of one Mamba3 mixer, everything between in_proj and out_proj
 * of Mamba3.step (layer.py:298-371) in one kernel: split of the in_proj row, softplus /
 * clamp / sigmoid, RMSNorm + bias of B and C, angle update and RoPE, the state update,
 * the C.h readout, the D skip, (MIMO) the rank projections, and the silu(z) gate.
 *   zxbcdt      (batch, d_in_proj) in_proj output, f32 / bf16 / f16
 *   dt_bias (H) f32;  B_bias, C_bias (H, R, D) f32;  B_norm_w, C_norm_w (D) f32;  Dskip (H) f32
 *   mimo_x, mimo_o (H, R, P) (MIMO only)
 *   angle_in/out (batch, H, S) f32;  ssm_in/out, bx_in/out: SISO (batch,H,P,D), MIMO (batch,H,D) f32
 *               (an output may alias its input: the update is then in place)
 *   y_gated     (batch, d_inner), dtype of zxbcdt: y * silu(z), the out_proj input.
 * ------------------------------------------------------------------------------- */
int m3_siso_step(const m3_layer_dims* dims, const m3_tensor* zxbcdt, const m3_tensor* dt_bias,
                 const m3_tensor* B_bias, const m3_tensor* C_bias, const m3_tensor* B_norm_w,
                 const m3_tensor* C_norm_w, const m3_tensor* Dskip, const m3_tensor* angle_in,
                 const m3_tensor* ssm_in, const m3_tensor* bx_in, m3_tensor* angle_out,
                 m3_tensor* ssm_out, m3_tensor* bx_out, m3_tensor* y_gated, void* stream);

int m3_mimo_step(const m3_layer_dims* dims, const m3_tensor* zxbcdt, const m3_tensor* dt_bias,
                 const m3_tensor* B_bias, const m3_tensor* C_bias, const m3_tensor* B_norm_w,
                 const m3_tensor* C_norm_w, const m3_tensor* Dskip, const m3_tensor* mimo_x,
                 const m3_tensor* mimo_o, const m3_tensor* angle_in, const m3_tensor* ssm_in,
                 const m3_tensor* bx_in, m3_tensor* angle_out, m3_tensor* ssm_out,
                 m3_tensor* bx_out, m3_tensor* y_gated, void* stream);

/* ---------------------------------------------------------------------------------
 * RMSNorm with an optional fused residual add: the reference's RMSNorm.forward
 * (mamba3_ssm/ops.py:94-102, x.float() / sqrt(mean(x^2) + eps) * weight, returned in
 * x.dtype), used by MambaBlock (block.py:20-29, x + mixer(norm(x))), the B / C norms of
 * Mamba3 (layer.py:215-225) and norm_f (block.py:78-80).
 *   x, residual, out, residual_out: (..., d), one dtype (f32 / bf16 / f16), innermost
 *   stride 1, leading dims collapsible into rows of one stride
 *   weight (d) f32 / bf16 / f16
 * With residual: h = x + residual (rounded to x.dtype like the eager add) is written to
 * residual_out (optional; may alias x) and normalised. out may alias x or residual, not
 * residual_out. Stream-ordered; the reference has no native counterpart (plain PyTorch).
 * ------------------------------------------------------------------------------- */
int m3_rmsnorm(const m3_tensor* x, const m3_tensor* residual, const m3_tensor* weight, float eps,
               m3_tensor* out, m3_tensor* residual_out, void* stream);

/* ---------------------------------------------------------------------------------
 * Greedy token choice of the decode step: out[r] = argmax over the last dimension of
 * logits[r] (the logits.argmax(-1) of greedy decoding with MambaLMHeadModel, block.py /
 * generate: first index of the maximum, NaN counting as the maximum, like torch.argmax).
 *   logits (..., n) f32 / bf16 / f16, innermost stride 1, leading dims collapsible into
 *   rows of one stride; out: int64, contiguous, one element per row.
 * No counterpart in the reference's native code (a PyTorch reduction there).
 * ------------------------------------------------------------------------------- */
int m3_argmax_rows(const m3_tensor* logits, m3_tensor* out, void* stream);

/* ---------------------------------------------------------------------------------
 * Fused forward prologue of Mamba3.forward (layer.py:180-244) for inference, from the
 * in_proj output zxbcdt (batch, seqlen, d_in_proj) (innermost stride 1, any dtype):
 *   DT = softplus(dd_dt + dt_bias), ADT = -min(softplus(dd_A), -A_floor) * DT, trap = the
 *   logit in fp32 (all (batch, seqlen, nheads) fp32 contiguous); angles (batch, seqlen,
 *   nheads, num_rope_angles) fp32 = cumsum over seqlen of angle_raw * DT; B_proj, C_proj
 *   (batch, seqlen, mimo_rank, nheads, d_state) contiguous, f32 / bf16 / f16: RMSNorm
 *   (eps = dims->norm_eps) * weight + bias per head, pairs (2i, 2i+1) with 2i < rope_split
 *   rotated by angles. Parameters fp32 as in m3_siso_step. Replaces the PyTorch prologue
 *   of the reference (layer.py:198-244), which materialises the per-head B / C in fp32.
 *   angle0 (batch, nheads, S) f32, optional: the angle state of a decode cache to continue
 *   from (the cumulative angles then start there, as they would after that many step()s);
 *   absent = zeros, as in the reference's forward.
 *   B_proj and C_proj may both be NULL: only ADT, DT, trap and angles are written (the
 *   inputs of m3_mimo_layer_scan_fwd, which forms B / C itself).
 * ------------------------------------------------------------------------------- */
int m3_layer_prologue(const m3_layer_dims* dims, const m3_tensor* zxbcdt, const m3_tensor* dt_bias,
                      const m3_tensor* B_bias, const m3_tensor* C_bias, const m3_tensor* B_norm_w,
                      const m3_tensor* C_norm_w, const m3_tensor* angle0, m3_tensor* B_proj,
                      m3_tensor* C_proj, m3_tensor* ADT, m3_tensor* DT, m3_tensor* trap,
                      m3_tensor* angles, void* stream);

/* ---------------------------------------------------------------------------------
 * MIMO scan of one Mamba3 layer straight from its in_proj output, for inference with one
 * B / C group (ngroups 1): the per-head B / C of layer.py:214-244 (RMSNorm of the group
 * rows * weight + per-head bias, pairs rotated by the angles) are formed inside the scan
 * and never written, then the scan of ssm_scan_mimo (ops.py:184-242) and, with gate = 1,
 * the gate y * silu(z) of layer.py:262-266. Equals m3_layer_prologue's B_proj / C_proj
 * followed by m3_mimo_scan_fwd_ws and m3_silu_gate, up to rounding (B / C stay fp32 here).
 *   zxbcdt (batch, seqlen, d_in_proj) f32 / bf16 / f16, innermost stride 1: z, x and the
 *   group rows are read from it; its start, row strides, 2 * d_inner, headdim and d_state
 *   in whole 16-byte units;
 *   ADT, DT, trap (batch, seqlen, nheads) f32 and angles (batch, seqlen, nheads, S) f32
 *   contiguous: m3_layer_prologue's outputs (B_proj / C_proj may be NULL there);
 *   B_bias, C_bias (nheads, rank, d_state), B_norm_w, C_norm_w (d_state) f32 contiguous,
 *   16-byte aligned; D (nheads), mimo_x, mimo_o (nheads, rank, headdim) f32;
 *   h0, bx0 (batch, nheads, d_state) f32 optional: states to continue from;
 *   out (batch, seqlen, nheads, headdim), zxbcdt's dtype: y, or y * silu(z) with gate = 1;
 *   h_last, bx_last optional, as in m3_mimo_scan_fwd;
 *   workspace: m3_mimo_scan_fwd_workspace_size(...) bytes, 16-byte aligned.
 * M3_ERR_UNSUPPORTED (nothing launched) when ngroups > 1 or the layout does not allow
 * the kernel's TMA boxes; the caller then runs m3_layer_prologue with B_proj / C_proj and
 * m3_mimo_scan_fwd_ws. Replaces the PyTorch prologue of layer.py:214-244, whose per-head
 * B / C are (batch, seqlen, rank, nheads, d_state) fp32 tensors, and the scan call.
 * ------------------------------------------------------------------------------- */
int m3_mimo_layer_scan_fwd(const m3_layer_dims* dims, const m3_tensor* zxbcdt, const m3_tensor* ADT,
                           const m3_tensor* DT, const m3_tensor* trap, const m3_tensor* angles,
                           const m3_tensor* B_bias, const m3_tensor* C_bias, const m3_tensor* B_norm_w,
                           const m3_tensor* C_norm_w, const m3_tensor* D, const m3_tensor* mimo_x,
                           const m3_tensor* mimo_o, const m3_tensor* h0, const m3_tensor* bx0, int32_t gate,
                           m3_tensor* out, m3_tensor* h_last, m3_tensor* bx_last, void* workspace,
                           size_t workspace_bytes, void* stream);

/* out = y * silu(z), (B, L, H, P) views with innermost stride 1; the gate of
 * Mamba3.forward between the scan and out_proj (layer.py:262-266). */
int m3_silu_gate(const m3_tensor* y, const m3_tensor* z, m3_tensor* out, void* stream);

/* ---------------------------------------------------------------------------------
 * Backward of the prologue and of the gate, for training (the gradients autograd returns
 * through layer.py:198-266; the reference differentiates its PyTorch prologue).
 * m3_layer_prologue_bwd: from the forward's in_proj output zxbcdt, DT and angles (as
 *   m3_layer_prologue wrote them) and the scan's gradients dB_proj / dC_proj (batch,
 *   seqlen, R, H, D, the scan operand dtype), dADT, dDT, dtrap (batch, seqlen, H) f32,
 *   writes the B, C, dt, A (zeros: the clamp of layer.py:207 passes no gradient), trap and
 *   angle columns of d_zxbcdt (zxbcdt's shape and dtype; the z and x columns are left to
 *   m3_silu_gate_bwd and the scan backward) and overwrites the parameter gradients
 *   d_dt_bias (H), d_B_bias / d_C_bias (H, R, D), d_B_norm_w / d_C_norm_w (D), all f32.
 *   workspace: m3_layer_prologue_bwd_workspace_size bytes, 16-byte aligned.
 * m3_silu_gate_bwd: dy = dout * silu(z), dz = dout * y * silu'(z), all (B, L, H, P) views of
 *   one dtype with innermost stride 1.
 * ------------------------------------------------------------------------------- */
size_t m3_layer_prologue_bwd_workspace_size(const m3_layer_dims* dims, int64_t batch, int64_t seqlen);
int m3_layer_prologue_bwd(const m3_layer_dims* dims, const m3_tensor* zxbcdt, const m3_tensor* dt_bias,
                          const m3_tensor* B_bias, const m3_tensor* C_bias, const m3_tensor* B_norm_w,
                          const m3_tensor* C_norm_w, const m3_tensor* DT, const m3_tensor* angles,
                          const m3_tensor* dB_proj, const m3_tensor* dC_proj, const m3_tensor* dADT,
                          const m3_tensor* dDT, const m3_tensor* dtrap, m3_tensor* d_zxbcdt,
                          m3_tensor* d_dt_bias, m3_tensor* d_B_bias, m3_tensor* d_C_bias,
                          m3_tensor* d_B_norm_w, m3_tensor* d_C_norm_w, void* workspace,
                          size_t workspace_bytes, void* stream);
int m3_silu_gate_bwd(const m3_tensor* y, const m3_tensor* z, const m3_tensor* dout, m3_tensor* dy,
                     m3_tensor* dz, void* stream);

/* ---------------------------------------------------------------------------------
 * Health word of the warp-specialised kernels and of the single-pass MIMO forward on the
 * current device: *flag_out is nonzero once any bounded wait (between warps, on a TMA
 * box, or on an earlier chunk's published state) gave up (the kernel then drained and its
 * outputs are invalid); reset != 0 clears it. Synchronises the device. No reference
 * counterpart (the reference checks no launch at all, cuda_backend.py:403-405).
 * ------------------------------------------------------------------------------- */
int m3_device_timeouts(int reset, int* flag_out);

#ifdef __cplusplus
}
#endif

#endif /* MAMBA3_B200_H */
