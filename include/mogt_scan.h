/* mogt_scan.h — C ABI of the B200 (sm_100a) MOGT scan library, libmogt_scan.so.
 *
 * The library computes MOGT's affine recurrence H_t = U_t H_{t-1} + V_t and
 * its headed, gated form
 *     S_t = f_t S_{t-1} + (1 - f_t) k_t v_t^T,     o_t = S_t^T q_t
 * (U_t = f_t I, V_t = (1-f_t) k_t v_t^T), forward and backward.
 *
 * Conventions shared by every entry point:
 *   - all tensor pointers are DEVICE pointers of dense, C-contiguous arrays;
 *   - `stream` is a cudaStream_t (NULL = legacy default stream); every call is
 *     stream-ordered and asynchronous: no host synchronisation, no allocation;
 *   - the caller owns every buffer, including the `workspace` whose size the
 *     matching *_workspace_bytes() returns.  A workspace must be zero-filled
 *     once before its first use; each call leaves it ready for the next call.
 *     Calls that share a workspace must not overlap on the GPU (use one
 *     workspace per stream);
 *   - return value: MOGT_OK or one of the MOGT_ERR_* codes below.  Kernel-side
 *     failures (a look-back wait that timed out) are recorded in the
 *     workspace and read back with mogt_workspace_status().
 *
 * The reference (lkcfqy/MOGT) exposes this path as Python functions only; the
 * comment above each entry point names the reference function it replaces.
 */
#ifndef MOGT_SCAN_H_
#define MOGT_SCAN_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MOGT_ABI_VERSION 2

enum mogt_status {
  MOGT_OK = 0,
  MOGT_ERR_SHAPE = 1,       /* bad rank/shape: the reference raises ValueError */
  MOGT_ERR_DTYPE = 2,       /* unsupported dtype combination */
  MOGT_ERR_ALIGN = 3,       /* pointer not 16-byte aligned */
  MOGT_ERR_LAUNCH = 4,      /* CUDA launch / TMA descriptor failure */
  MOGT_ERR_TIMEOUT = 5,     /* a bounded device-side wait gave up */
  MOGT_ERR_WORKSPACE = 6,   /* workspace missing or too small */
  MOGT_ERR_UNSUPPORTED = 7, /* valid request this build does not implement */
  MOGT_ERR_ARG = 8,         /* null pointer where one is required */
  MOGT_ERR_TOO_LARGE = 9    /* problem needs more scratch than the fixed
                               buffer of mogt_gated_scan_fwd_noalloc */
};

enum mogt_dtype { MOGT_DTYPE_F32 = 0, MOGT_DTYPE_BF16 = 1, MOGT_DTYPE_F16 = 2 };

int mogt_abi_version(void);
const char* mogt_status_string(int status);

/* Copy the workspace's sticky error word to the host (synchronises `stream`).
 * *err_out = MOGT_OK or MOGT_ERR_TIMEOUT; *unit_out = first failing unit. */
int mogt_workspace_status(const void* workspace, void* stream, int* err_out, uint32_t* unit_out);
/* Zero a workspace (first use, or after an error). */
int mogt_workspace_clear(void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Headed gated scan, forward.  Replaces the composition the reference's MOGT
 * operator performs for a scalar gate: affine_scan.py:14-62
 * (affine_scan_sequential with U = f I, V = (1-f) k v^T) followed by the
 * readout einsum o_t = S_t^T q_t.
 *
 *   q, k : [BH, T, dk]   v, o : [BH, T, dv]   f : [BH, T] fp32
 *   in_dtype  : MOGT_DTYPE_BF16 (tensor-core chunked path, dk = dv = 64) or
 *               MOGT_DTYPE_F32 (exact fp32 path, dk, dv <= 128)
 *   out_dtype : dtype of o (MOGT_DTYPE_BF16 or MOGT_DTYPE_F32)
 *   S0          [BH, dk, dv] fp32 initial state, or NULL for zeros
 *   S_final     [BH, dk, dv] fp32 final state S_T, or NULL
 *   decay_final [BH] fp32 product of all f (the carry's decay), or NULL
 *   chunk_states [BH, nchunks, dk, dv] bf16 state entering each 64-step chunk
 *               (saved for the backward; bf16 path only), or NULL;
 *               nchunks = mogt_gated_scan_num_chunks()
 *   o may be NULL: only the final state / decay are produced (the first phase
 *   of the sequence-parallel scan).
 * Gates must lie in [0, 1] (the chunked path works with log2 f).
 * ------------------------------------------------------------------------- */
int64_t mogt_gated_scan_num_chunks(int64_t T, int64_t dk, int64_t dv, int in_dtype);
size_t mogt_gated_scan_fwd_workspace_bytes(int64_t BH, int64_t T, int64_t dk, int64_t dv,
                                           int in_dtype);
int mogt_gated_scan_fwd(const void* q, const void* k, const void* v, const float* f, void* o,
                        const float* S0, float* S_final, float* decay_final, void* chunk_states,
                        int64_t BH, int64_t T, int64_t dk, int64_t dv, int in_dtype, int out_dtype,
                        void* workspace, size_t workspace_bytes, void* stream);

/* Second half of a bf16 forward whose first half already ran: the segment
 * carry from the initial state S0 and the output pass, reusing the chunk-local
 * states that an earlier mogt_gated_scan_fwd call with the same k, v, f, BH,
 * T and workspace left there (that call may be state-only, o = NULL, and must
 * have been made with chunk_states = NULL; nothing may use the workspace in
 * between).  The sequence-parallel scan uses it: each rank's state-only pass
 * gives its segment carry, and after the carries are exchanged the output
 * pass resumes from the incoming state without re-reading k, v for the local
 * states.  Arguments as mogt_gated_scan_fwd; in_dtype must be MOGT_DTYPE_BF16.
 * Replaces the second full forward of the segment (the reference has no
 * sequence-parallel path; its carry algebra is affine_scan.py:250-271). */
int mogt_gated_scan_fwd_resume(const void* q, const void* k, const void* v, const float* f,
                               void* o, const float* S0, float* S_final, float* decay_final,
                               void* chunk_states, int64_t BH, int64_t T, int64_t dk, int64_t dv,
                               int in_dtype, int out_dtype, void* workspace,
                               size_t workspace_bytes, void* stream);

/* Allocation-free variant of mogt_gated_scan_fwd.  This entry point has no
 * counterpart in the reference.  It exists for callers that cannot allocate
 * device memory: hosts whose device memory is owned by an allocator or a
 * budget this library cannot reach through a C ABI (a runtime that reserves
 * all of its GPU memory up front, a foreign-language binding without access
 * to the caller's allocator), and code that must not pay the implicit device
 * synchronisation of cudaMalloc/cudaFree.  Arguments and results are those
 * of mogt_gated_scan_fwd minus the workspace: the scan's scratch lives in a
 * 16 MiB array built into the library, which every GPU that loads the library
 * keeps for the life of the process (enough for BASELINE-sized problems such
 * as 12 heads x 32768 steps; larger requests return MOGT_ERR_TOO_LARGE and
 * do nothing; every argument is checked before the array is touched).
 * The current device must be the one that owns `stream` and the pointers.
 * The first call on a device looks up that device's copy of the array (make
 * it before any stream capture); no call allocates.  All calls share the one
 * array and each call clears the part that must start at zero, so calls
 * whose GPU work overlaps (other streams, other host threads) race and must
 * be serialised by the caller.  A device-side wait that gives up is recorded
 * in the array and kept until mogt_gated_scan_fwd_noalloc_status reads it. */
int mogt_gated_scan_fwd_noalloc(const void* q, const void* k, const void* v, const float* f,
                                void* o, const float* S0, float* S_final, float* decay_final,
                                void* chunk_states, int64_t BH, int64_t T, int64_t dk, int64_t dv,
                                int in_dtype, int out_dtype, void* stream);

/* Status of the allocation-free entry point on the current device: waits for
 * `stream`, then *err_out = MOGT_OK or MOGT_ERR_TIMEOUT (the first failure
 * since the last read) and *unit_out = the unit that recorded it; the record
 * is cleared by the read.  No counterpart in the reference. */
int mogt_gated_scan_fwd_noalloc_status(void* stream, int* err_out, uint32_t* unit_out);

/* ---------------------------------------------------------------------------
 * Headed gated scan, backward: gradients of L = sum_t <o_t, do_t>.
 * Replaces the reference's backward for this operator, affine_scan.py:65-124
 * (affine_scan_sequential_backward: Sigma_t = g_t + U_{t+1}^T Sigma_{t+1},
 * dU_t = Sigma_t H_{t-1}^T), chained through U = f I, V = (1-f) k v^T and the
 * readout (g_t = q_t do_t^T).
 *   inputs as mogt_gated_scan_fwd, d_o : [BH, T, dv] (same dtype as q)
 *   dq, dk : [BH, T, dk], dv : [BH, T, dv] in the input dtype; df : [BH, T] fp32
 *   dS0 : [BH, dk, dv] fp32 gradient of the initial state S0, or NULL
 *   in_dtype MOGT_DTYPE_F32: exact sequential kernels (dk, dv <= 128); S0 is
 *     the forward's initial state (or NULL), chunk_states must be NULL.
 *   in_dtype MOGT_DTYPE_BF16 (dk = dv = 64): reverse-time chunked tensor-core
 *     kernel; chunk_states = the bf16 per-chunk states written by
 *     mogt_gated_scan_fwd on the same inputs (they already hold S0, which is
 *     ignored); all bf16 pointers 16-byte aligned.
 * ------------------------------------------------------------------------- */
size_t mogt_gated_scan_bwd_workspace_bytes(int64_t BH, int64_t T, int64_t dk, int64_t dv,
                                           int in_dtype);
int mogt_gated_scan_bwd(const void* q, const void* k, const void* v, const float* f,
                        const void* d_o, const float* S0, const void* chunk_states, void* dq,
                        void* dk, void* dv, float* df, float* dS0, int64_t BH, int64_t T, int64_t dk_, int64_t dv_, int in_dtype,
                        void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Dense-transition headed scan:
 *     S_t = A_t S_{t-1} + (1 - f_t) k_t v_t^T,   o_t = S_t^T q_t.
 * Replaces affine_scan.py:14-62 (affine_scan_sequential on U = A,
 * V = (1-f) k v^T) followed by the readout einsum.
 *   A : [BH, T, d, d] fp32 (16-byte aligned), q, k, v, o : [BH, T, d],
 *   f : [BH, T] fp32; S0 / S_final : [BH, d, d] fp32 or NULL; o may be NULL.
 *   d in {16, 32, 64}; in_dtype bf16 or f32; out_dtype bf16 or f32 (f32 for
 *   f32 inputs).  fp32 arithmetic throughout.
 * ------------------------------------------------------------------------- */
int mogt_matrix_scan_fwd(const float* A, const void* q, const void* k, const void* v,
                         const float* f, void* o, const float* S0, float* S_final, int64_t BH,
                         int64_t T, int64_t d, int in_dtype, int out_dtype, void* stream);

/* Arithmetic of the chunked dense-transition kernels. */
enum mogt_matrix_mode {
  MOGT_MATRIX_FP32 = 0,   /* fp32 FMAs, round-to-nearest (default) */
  MOGT_MATRIX_TF32X3 = 1  /* tensor cores, three tf32 products per step (bf16
                             q/k/v only); faster, but the tensor core's
                             accumulation rounding is biased, so the error
                             grows linearly with T for norm-preserving A
                             (measured 4e-4 relative at T = 8192) */
};

/* Chunked form of mogt_matrix_scan_fwd for long sequences (d = 64 only),
 * with the same arguments, results and arithmetic (see `mode`) plus:
 *   status  : a zero-initialised 256-byte workspace header (the one the
 *             gated-scan workspaces start with); a device-side wait that
 *             gives up records MOGT_ERR_TIMEOUT there
 *             (mogt_workspace_status reads it);
 *   scratch : >= mogt_matrix_scan_chunked_scratch_bytes(BH, T, d) bytes,
 *             16-byte aligned, any contents.
 * T is split into 64-step chunks; every chunk's transition prefix products
 * and local state run in parallel (bf16 q/k/v: on the tensor cores, three
 * tf32 products per step for fp32-level accuracy; fp32 q/k/v: fp32 FMAs),
 * the chunk carries are composed per head, and o = o_local +
 * (P_t^T q_t)^T S_in is formed per chunk.  Any T >= 1.
 * No counterpart in the reference beyond affine_scan.py:14-62, which this
 * computes in another order. */
size_t mogt_matrix_scan_chunked_scratch_bytes(int64_t BH, int64_t T, int64_t d);
int mogt_matrix_scan_fwd_chunked(const float* A, const void* q, const void* k, const void* v,
                                 const float* f, void* o, const float* S0, float* S_final,
                                 int64_t BH, int64_t T, int64_t d, int in_dtype, int out_dtype,
                                 int mode, void* status, void* scratch, size_t scratch_bytes,
                                 void* stream);

/* ---------------------------------------------------------------------------
 * Dense-transition headed scan, backward: gradients of L = sum_t <o_t, do_t>
 * for mogt_matrix_scan_fwd_chunked (d = 64).  Replaces the reference's
 * backward for this operator, affine_scan.py:65-124
 * (affine_scan_sequential_backward on U = A, V = (1-f) k v^T; Sigma_t = g_t +
 * A_{t+1}^T Sigma_{t+1}, dA_t = Sigma_t S_{t-1}^T) chained through the readout
 * (g_t = q_t do_t^T).
 *   A, q, k, v, f : the forward's inputs; d_o : [BH, T, d] (q's dtype);
 *   saved   : the forward's `scratch` after that call (it holds each chunk's
 *             entering state and transition product), unchanged since;
 *   dA : [BH, T, d, d] fp32; dq, dk, dv : [BH, T, d] in the input dtype;
 *   df : [BH, T] fp32; dS0 : [BH, d, d] fp32 gradient of the initial state,
 *   or NULL;
 *   status  : a zero-initialised 256-byte workspace header (timeouts);
 *   scratch : >= mogt_matrix_scan_bwd_scratch_bytes(BH, T, d) bytes,
 *             16-byte aligned, any contents.
 * fp32 arithmetic (round-to-nearest FMAs) throughout; in_dtype bf16 or f32.
 * ------------------------------------------------------------------------- */
size_t mogt_matrix_scan_bwd_scratch_bytes(int64_t BH, int64_t T, int64_t d);
int mogt_matrix_scan_bwd(const float* A, const void* q, const void* k, const void* v,
                         const float* f, const void* d_o, const void* saved, float* dA, void* dq,
                         void* dk, void* dv, float* df, float* dS0, int64_t BH, int64_t T, int64_t d,
                         int in_dtype, void* status, void* scratch, size_t scratch_bytes,
                         void* stream);

/* ---------------------------------------------------------------------------
 * Diagonal gated scan with the RMSNorm readout fused: the MOGT block with the
 * identity connection and the forget gate coupled to the value gate
 * (model_mogt.py:168-182 gating, :225 scan, :240 norm_out).  Replaces, for
 * that configuration, U = damping (1 - z) I, V = V * z.to(V.dtype),
 * H = triton_affine_scan_hybrid(U, V) (triton_scan.py:429-477) and
 * norm_out(H):
 *   h_t = damping (1 - z_t[row]) h_{t-1} + v_t z_t[row]  per channel,
 *   y_t = h_t * rsqrt(mean(h_t^2) + eps) * norm_weight   per token.
 *   V : [B, L, R, C] bf16 or f32 (16-byte aligned); z : [B, L, z_per_token]
 *   f32 with z_per_token = R (row-wise gate) or 1 (one gate);
 *   H0 : [B, R, C] f32 initial state or NULL; norm_weight : [R*C] f32;
 *   y : [B, L, R*C] in out_dtype (bf16 or f32); H_final : [B, R, C] f32 or
 *   NULL.  C even, R*C a multiple of 64 and <= 2048, R <= 64.
 *   status  : a zero-initialised 256-byte workspace header; a device-side
 *             wait that gives up records MOGT_ERR_TIMEOUT there;
 *   scratch : >= mogt_diag_scan_norm_scratch_bytes(B, L, R, C, in_dtype)
 *             bytes, 16-byte aligned.
 * ------------------------------------------------------------------------- */
size_t mogt_diag_scan_norm_scratch_bytes(int64_t B, int64_t L, int64_t R, int64_t C,
                                         int in_dtype);
int mogt_diag_scan_norm_fwd(const void* V, const float* z, int64_t z_per_token, float damping,
                            const float* H0, const float* norm_weight, float eps, void* y,
                            float* H_final, int64_t B, int64_t L, int64_t R, int64_t C,
                            int in_dtype, int out_dtype, void* status, void* scratch,
                            size_t scratch_bytes, void* stream);

/* Backward of mogt_diag_scan_norm_fwd: gradients of L = sum <y, dy> with
 * respect to V, z, norm_weight and H0 (the chain rule the reference's
 * autograd takes through model_mogt.py:168-240 and affine_scan.py:65-124).
 *   V, z, z_per_token, damping, norm_weight, eps: the forward's arguments;
 *   dy : [B, L, R*C] in dy_dtype (bf16 or f32);
 *   fwd_scratch : the forward's `scratch` after that call (it holds the
 *             state entering each of the forward's chunks), unchanged since;
 *   dV : [B, L, R, C] in V's dtype; dz : [B, L, z_per_token] f32;
 *   d_norm_weight : [R*C] f32; dH0 : [B, R, C] f32 or NULL;
 *   scratch : >= mogt_diag_scan_norm_bwd_scratch_bytes(B, L, R, C) bytes.
 *   R*C <= 1024.  Reverse-time chunked (8-token chunks): chunk-local adjoint
 *   aggregates, the adjoint carry per channel, then the gradients. */
size_t mogt_diag_scan_norm_bwd_scratch_bytes(int64_t B, int64_t L, int64_t R, int64_t C);
int mogt_diag_scan_norm_bwd(const void* V, const float* z, int64_t z_per_token, float damping,
                            const float* norm_weight, float eps, const void* dy,
                            const void* fwd_scratch, void* dV, float* dz, float* d_norm_weight,
                            float* dH0, int64_t B, int64_t L, int64_t R, int64_t C, int in_dtype,
                            int dy_dtype, void* status, void* scratch, size_t scratch_bytes,
                            void* stream);

/* ---------------------------------------------------------------------------
 * Connection map of the MOGT block (replaces model_mogt.py:79-102,
 * _build_transport: torch.matrix_exp / torch.linalg.solve on [B, L, r, r]).
 * For each of `count` n x n matrices M (row-major, consecutive):
 *   A = (M - M^T) * scale         (skew != 0; the block's antisymmetrised
 *                                  phi_conn output, scale = 1 / r)
 *   A = M                         (skew == 0)
 *   U = damping * expm(A)                         mode MOGT_CONN_EXPM
 *   U = damping * (I - A/2)^{-1} (I + A/2)        mode MOGT_CONN_CAYLEY
 * fp32 arithmetic; M in_dtype, U out_dtype (f32 or bf16); n in {8, 16, 32}.
 * ------------------------------------------------------------------------- */
enum mogt_conn_mode { MOGT_CONN_EXPM = 0, MOGT_CONN_CAYLEY = 1 };
int mogt_connection_map(const void* M, void* U, int64_t count, int64_t n, int mode, int skew,
                        float scale, float damping, int in_dtype, int out_dtype, void* stream);

/* ---------------------------------------------------------------------------
 * Softmax cross-entropy rows of the chunked linear cross-entropy (replaces the
 * F.cross_entropy / softmax steps of chunked_lm_loss.py:25-35, 52-61).
 *   logits : [rows, V] fp32 (one chunk's hidden @ weight^T), 16-byte aligned
 *            rows when V % 4 == 0 for the vector path;
 *   labels : [rows] int64 in [0, V) or -100 (ignored by the loss);
 *   fwd: lse[i] = log sum_j exp(logits[i, j]); loss[i] = lse[i] -
 *        logits[i, labels[i]] (0 for -100);
 *   bwd: in place, logits[i, j] = (exp(logits[i, j] - lse[i]) - [j == l_i]) *
 *        scale with l_i = labels[i] (+ V when negative, as the reference's
 *        indexing does).
 * ------------------------------------------------------------------------- */
int mogt_ce_rows_fwd(const float* logits, const int64_t* labels, int64_t rows, int64_t V, float* lse,
                     float* loss, void* stream);
int mogt_ce_rows_bwd(float* logits, const int64_t* labels, const float* lse, int64_t rows, int64_t V,
                     float scale, void* stream);

/* ---------------------------------------------------------------------------
 * Dense affine scan H_t = U_t H_{t-1} + V_t, H_{-1} = 0 (fp32 state).
 * Replaces triton_scan.py:232-311 (_triton_affine_scan_hybrid_forward: local
 * Triton kernel + Python carry scan + carry apply), triton_scan.py:151-175
 * (triton_fused_scan: C = 0, prefix products only) and the reverse scan of
 * triton_scan.py:398-416 / affine_scan.py:110-118 (reverse != 0).
 *
 *   U : [B, L, R, R] (f32 or bf16),  V : [B, L, R, C] (f32 or bf16)
 *   H : [B, L, R, C] out_dtype, the states H_t; may be NULL when C == 0
 *   U_prefix : [B, L, R, R] out_dtype, P_t = U_t ... U_0, or NULL
 *   reverse != 0 computes Sigma_t = V_t + U_{t+1}^T Sigma_{t+1} (the adjoint
 *   recurrence of the backward, V = grad_H) into H; U_prefix must be NULL.
 *   R in {2, 4, 8, 16, 32}; C + R <= 512 (R <= 16) or <= 256 (R = 32).
 * ------------------------------------------------------------------------- */
size_t mogt_affine_scan_workspace_bytes(int64_t B, int64_t L, int64_t R, int64_t C);
int mogt_affine_scan_fwd(const void* U, const void* V, void* H, void* U_prefix, int64_t B,
                         int64_t L, int64_t R, int64_t C, int u_dtype, int v_dtype, int out_dtype,
                         int reverse, void* workspace, size_t workspace_bytes, void* stream);

/* dU_t = Sigma_t H_{t-1}^T with H_{-1} = 0 (affine_scan.py:117 /
 * triton_scan.py:421-424).  sigma, H : [B, L, R, C] fp32; grad_U : [B, L, R, R]
 * in out_dtype. */
int mogt_affine_grad_u(const float* sigma, const float* H, void* grad_U, int64_t B, int64_t L,
                       int64_t R, int64_t C, int out_dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MOGT_SCAN_H_ */
