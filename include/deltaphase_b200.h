/*
 * deltaphase_b200.h -- C ABI of the B200 (sm_100a) DeltaPhase inference kernels.
 *
 * Every entry point takes plain device pointers, sizes, element strides and a
 * cudaStream_t passed as `void *` (NULL = legacy default stream), launches
 * asynchronously on that stream, allocates nothing and returns an int status
 * (DP_OK = 0).  On failure dp_last_error() returns a message for the calling
 * host thread.  No entry point synchronises the stream.
 *
 * Conventions shared by all entry points
 *   - dtype codes: DP_F32, DP_BF16, DP_F16 for phase / value / beta / x inputs.
 *   - Complex states (the reference's complex64 M of shape (B, H, Dv, D), row =
 *     value channel, column = key channel) are passed as float pointers to the
 *     interleaved (re, im) pairs, i.e. torch.view_as_real(M), contiguous.
 *   - Strides are in elements.  Sequence tensors are addressed as
 *     base + b*sb + h*sh + t*st + c with unit stride over the channel c, so the
 *     (B, L, H, D) projection outputs of a block can be passed without a copy.
 *
 * Reference: mcarbonell/delta-phase v1.3.0 (pure PyTorch); each declaration
 * names the reference interface it replaces.
 */
#ifndef DELTAPHASE_B200_H
#define DELTAPHASE_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define DP_API __attribute__((visibility("default")))
#else
#define DP_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum dp_dtype { DP_F32 = 0, DP_BF16 = 1, DP_F16 = 2 };

enum dp_status {
  DP_OK = 0,
  DP_ERR_INVALID_ARGUMENT = 1, /* null pointer, negative size, bad dtype code  */
  DP_ERR_UNSUPPORTED = 2,      /* shape outside the kernel's limits            */
  DP_ERR_MISALIGNED = 3,       /* pointer/stride alignment a kernel requires   */
  DP_ERR_CUDA = 4,             /* launch or runtime error reported by CUDA     */
  DP_ERR_TIMEOUT = 5,          /* a device-side wait exceeded its bound        */
  DP_ERR_WORKSPACE = 6,        /* workspace too small                          */
  DP_ERR_RANGE = 7             /* a value left the range of a kernel's 16-bit
                                  operand tiles (reported by dp_device_error)   */
};

/* Library version string, e.g. "deltaphase_b200 0.1.0 (sm_100a)". */
DP_API const char *dp_version(void);
/* Message of the last failed call made by this host thread ("" if none). */
DP_API const char *dp_last_error(void);
/* Name of a status code. */
DP_API const char *dp_status_string(int status);
/* Synchronises the current device and returns the device-side error word (0, or
 * DP_ERR_TIMEOUT if a kernel's bounded wait expired, DP_ERR_RANGE if an operand left
 * the fp16 range of dp_core_cbeta_fwd's tensor-core tiles, since the last clear); clears
 * it when `clear` is non-zero.  Returns -1 if the CUDA runtime reports an error. */
DP_API int dp_device_error(int clear);

/*
 * Chunkwise complex delta-rule forward (inference).
 * Replaces _chunkwise_delta_reference / delta_phase_chunkwise_fused
 * (delta_phase/kernels/triton_chunk_delta.py:211-252, :279-291) and the core
 * inlined in DeltaPhaseHolographicBlock.forward (delta_phase/layers.py:203-236).
 *
 *   theta_k, theta_q : (B, H, L, D)  phases, dtype in_dtype
 *   v                : (B, H, L, Dv) values, dtype in_dtype
 *   beta             : (B, H, L)     write strengths, dtype beta_dtype
 *   state_in         : (B, H, Dv, D) complex64 initial state or NULL (= zero)
 *   out              : (B, H, L, Dv) float32 retrieved values
 *   state_out        : (B, H, Dv, D) complex64 final state (may equal state_in)
 *   strides[15]      : {sb, sh, st} of theta_k, theta_q, v, beta, out (beta's
 *                      st is its token stride)
 * Any L >= 0 is accepted; the result equals the reference's chunkwise path for
 * every chunk_size (>= 1) because it is the same recurrence -- the kernel picks
 * its own internal chunking.  Limits: 1 <= D, Dv <= 128.
 */
DP_API int dp_core_fwd(const void *theta_k, const void *theta_q, const void *v, const void *beta,
                int in_dtype, int beta_dtype, const float *state_in, float *out,
                float *state_out, int B, int H, int L, int D, int Dv, int chunk_size,
                const int64_t *strides, void *stream);

/*
 * Backward of the chunkwise core (training): gradients with respect to theta_k, theta_q,
 * v, beta and the initial state, given grad_out = dL/d out and grad_state_out = dL/dM
 * (or NULL = 0).  The reference trains through autograd of its PyTorch chunkwise path
 * (delta_phase/kernels/triton_chunk_delta.py:211-252, dispatched at :279-291; its
 * DeltaPhaseTritonFunction.backward, :271-276, raises) and of the complex-beta token loop
 * (delta_phase/layers.py:346-360); this is the adjoint of the same recurrence, in fp32.
 *
 *   theta_k, theta_q, v, beta : as dp_core_fwd (complex_beta != 0: beta holds phi, the
 *                               gradient written is d phi)
 *   state_in                  : (B, H, Dv, D) complex64 initial state or NULL (= zero)
 *   grad_out                  : (B, H, L, Dv) float32, contiguous
 *   grad_state_out            : (B, H, Dv, D) complex64 (as interleaved floats) or NULL
 *   grad_theta_k, grad_theta_q: (B, H, L, D) float32, contiguous
 *   grad_v                    : (B, H, L, Dv) float32, contiguous
 *   grad_beta                 : (B, H, L) float32, contiguous
 *   grad_state_in             : (B, H, Dv, D) complex64 (as floats) or NULL
 *   strides[12]               : {sb, sh, st} of theta_k, theta_q, v, beta
 *   workspace                 : dp_core_bwd_workspace_size(B, H, L, Dv) bytes
 * Complex gradients follow PyTorch's convention (dL/dRe + i dL/dIm).  Limits:
 * 1 <= D, Dv <= 64.
 */
DP_API size_t dp_core_bwd_workspace_size(int B, int H, int L, int Dv);
DP_API int dp_core_bwd(const void *theta_k, const void *theta_q, const void *v, const void *beta,
                int in_dtype, int beta_dtype, int complex_beta, const float *state_in,
                const float *grad_out, const float *grad_state_out, float *grad_theta_k,
                float *grad_theta_q, float *grad_v, float *grad_beta, float *grad_state_in,
                int B, int H, int L, int D, int Dv, const int64_t *strides, void *workspace,
                size_t workspace_bytes, void *stream);

/*
 * Phasors e^{i theta} = cos theta + i sin theta of n phases, written as interleaved
 * complex64 (out[2i] = cos, out[2i+1] = sin).  The elementwise step of
 * DeltaPhaseHolographicBlock.forward/step (delta_phase/layers.py:203-206, 275-278) and
 * of _chunkwise_delta_reference (delta_phase/kernels/triton_chunk_delta.py:220-221);
 * the fused kernels compute the same values in registers.  Max abs error ~2e-6 for
 * |theta| <= 20 (FMA-pipe Cody-Waite reduction + Taylor series).
 */
DP_API int dp_phasor(const void *theta, int dtype, int64_t n, float *out, void *stream);

/*
 * Single-token decode step: v_old = Re(M conj(k))/D; M += beta (v - v_old) k^T;
 * out = Re(M conj(q))/D (read after the update).
 * Replaces the state update of DeltaPhaseHolographicBlock.step
 * (delta_phase/layers.py:279-285) and the never-launched
 * _triton_streaming_step_kernel (delta_phase/kernels/triton_chunk_delta.py:125-185).
 *
 *   state_in/state_out : (B, H, Dv, D) complex64; may alias (in-place update)
 *   theta_k, theta_q   : (B, H, D);  v : (B, H, Dv);  beta : (B, H)
 *   out                : (B, H, Dv) float32
 *   strides[10]        : {sb, sh} of theta_k, theta_q, v, beta, out
 */
DP_API int dp_core_decode(const float *state_in, float *state_out, const void *theta_k,
                   const void *theta_q, const void *v, const void *beta, int in_dtype,
                   int beta_dtype, float *out, int B, int H, int D, int Dv,
                   const int64_t *strides, void *stream);

/*
 * Complex-beta (Householder) variants: beta_t = 1 + e^{i phi_t} per (b, h, t), the
 * update M += beta (v - Re(M conj(k))/D) k^T of ComplexBetaDeltaPhaseBlock
 * (delta_phase/layers.py:294-418).  The reference runs it as a token loop
 * (forward, layers.py:346-360; step, :402-407); dp_core_cbeta_fwd is its chunkwise
 * (WY) form, dp_core_cbeta_decode one step.  Arguments, layouts, strides and limits are
 * those of dp_core_fwd / dp_core_decode with `phi` (B, H, L) resp. (B, H) in place of
 * beta; phi_dtype is its dtype code.
 */
DP_API int dp_core_cbeta_fwd(const void *theta_k, const void *theta_q, const void *v, const void *phi,
                int in_dtype, int phi_dtype, const float *state_in, float *out,
                float *state_out, int B, int H, int L, int D, int Dv, int chunk_size,
                const int64_t *strides, void *stream);
DP_API int dp_core_cbeta_decode(const float *state_in, float *state_out, const void *theta_k,
                   const void *theta_q, const void *v, const void *phi, int in_dtype,
                   int phi_dtype, float *out, int B, int H, int D, int Dv,
                   const int64_t *strides, void *stream);

/*
 * Decode step that reads the write gate's raw projection and forms the gate itself,
 * so a block's step needs no separate gate kernels:
 *   DP_GATE_BETA     beta = gate                 (dp_core_decode)
 *   DP_GATE_SIGMOID2 beta = 2 sigmoid(gate)      (w_beta gate, delta_phase/layers.py:195, 265)
 *   DP_GATE_ONE      beta = 1, gate not read (may be NULL)  (beta_mode "fixed", layers.py:196-197, 266-267)
 *   DP_GATE_PHI      beta = 1 + e^{i gate}       (dp_core_cbeta_decode, layers.py:397-398)
 * Arguments otherwise as dp_core_decode; gate_dtype is the gate's dtype code.
 */
enum dp_gate_mode { DP_GATE_BETA = 0, DP_GATE_SIGMOID2 = 1, DP_GATE_ONE = 2, DP_GATE_PHI = 3 };
DP_API int dp_core_decode_gated(const float *state_in, float *state_out, const void *theta_k,
                   const void *theta_q, const void *v, const void *gate, int in_dtype,
                   int gate_dtype, int gate_mode, float *out, int B, int H, int D, int Dv,
                   const int64_t *strides, void *stream);

/*
 * Strictly-lower, row-beta-scaled phasor Gram of N chunks:
 *   G[n, m, j] = beta[n, m] * sum_d cos(theta[n,m,d] - theta[n,j,d]) / D  (m > j), else 0.
 * Replaces gram_matrix_triton / _triton_fused_phase_gram_kernel
 * (delta_phase/kernels/triton_chunk_delta.py:32-122); contract of
 * gram_matrix_reference (:192-208).  theta (N, C, D), beta (N, C), out (N, C, C)
 * float32, all contiguous.  Limits: C <= 256, D <= 256.
 */
DP_API int dp_gram(const void *theta, const void *beta, int in_dtype, int beta_dtype, float *out,
            int N, int C, int D, void *stream);

/*
 * LaplacePhaseCore chunkwise forward with per-row decay.
 * Replaces the chunk loop of LaplacePhaseCore.forward (delta_phase/layers.py:481-561),
 * fed the outputs of _project (layers.py:462-479):
 *   K = exp(logmag_k) e^{i theta_k},  Q = exp(logmag_q) e^{i theta_q},
 *   r = exp(log_decay) per (token, value channel), clamped like the reference
 *   (log r >= -80, layers.py:445,512).
 * Recurrence: v_old = Re(M conj(k_t))/D (pre-decay); M = diag(r_t) M + beta_t (v_t - v_old) k_t^T;
 * out_t = Re(M conj(q_t))/D.
 *   theta_k, theta_q, logmag_k, logmag_q : (B, H, L, D) (logmag_* may be NULL = 0)
 *   v, log_decay : (B, H, L, Dv);  beta : (B, H, L)
 *   strides[24]  : {sb, sh, st} of theta_k, logmag_k, theta_q, logmag_q, v,
 *                  log_decay, beta, out (entries of NULL tensors are ignored)
 * Limits: 1 <= D, Dv <= 128.
 */
DP_API int dp_laplace_fwd(const void *theta_k, const void *logmag_k, const void *theta_q,
                   const void *logmag_q, const void *v, const void *log_decay,
                   const void *beta, int in_dtype, int beta_dtype, const float *state_in,
                   float *out, float *state_out, int B, int H, int L, int D, int Dv,
                   int chunk_size, const int64_t *strides, void *stream);

/*
 * Backward of dp_laplace_fwd (training): gradients with respect to theta_k, logmag_k,
 * theta_q, logmag_q, v, log_decay, beta and the initial state, given grad_out = dL/d out
 * and grad_state_out = dL/dM (or NULL = 0).  The reference trains LaplacePhaseCore through
 * autograd of its chunk loop (delta_phase/layers.py:481-561); this is the adjoint of the
 * same recurrence in fp32 (log r clamped at -80 like the forward, zero gradient there).
 *   inputs, dtypes, strides[21] : as dp_laplace_fwd without `out` ({sb, sh, st} of
 *                                 theta_k, logmag_k, theta_q, logmag_q, v, log_decay, beta)
 *   grad_out                    : (B, H, L, Dv) float32, contiguous
 *   grad_theta_k/logmag_k/theta_q/logmag_q : (B, H, L, D) float32, contiguous
 *   grad_v, grad_log_decay      : (B, H, L, Dv) float32;  grad_beta : (B, H, L) float32
 *   grad_state_in               : (B, H, Dv, D) complex64 as floats, or NULL
 *   workspace                   : dp_laplace_bwd_workspace_size(B, H, L, D, Dv) bytes
 * Limits: 1 <= D, Dv <= 64.
 */
DP_API size_t dp_laplace_bwd_workspace_size(int B, int H, int L, int D, int Dv);
DP_API int dp_laplace_bwd(const void *theta_k, const void *logmag_k, const void *theta_q,
                   const void *logmag_q, const void *v, const void *log_decay, const void *beta,
                   int in_dtype, int beta_dtype, const float *state_in, const float *grad_out,
                   const float *grad_state_out, float *grad_theta_k, float *grad_logmag_k,
                   float *grad_theta_q, float *grad_logmag_q, float *grad_v, float *grad_log_decay,
                   float *grad_beta, float *grad_state_in, int B, int H, int L, int D, int Dv,
                   const int64_t *strides, void *workspace, size_t workspace_bytes, void *stream);

/*
 * Fold the spectral Lerp FFN parameters into one (6d x d) matrix.
 * With a_b = cos(h_b + phi1_b) w1_b + sin(h_b + phi2_b) w2_b
 *           = cos(h_b) alpha_b + sin(h_b) gamma_b   (angle addition), the FFN of
 * LearnableSubstrateLerpFFN.forward (delta_phase/layers.py:119-141) is exactly
 *   y = sum_b softmax(logits)_b (a_b W_c^T) M_b = z F,
 *   z = [cos h_fwht, sin h_fwht, cos h_dct, sin h_dct, cos h_haar, sin h_haar],
 *   F[(2b+s) d + i, j] = w_b sum_m (sum_k coef_{b,s}[k,i] W_c[m, k d + i]) M_b[m, j].
 * Inputs (float32, contiguous): logits (3); mats (3, d, d) = mat_fwht, mat_dct,
 * mat_haar; banks (3, 4, nb, d) = per branch {phi1, phi2, w1, w2}; combine
 * (d, nb*d).  Output F (6d, d) float32.  Accumulates in float64.
 */
DP_API int dp_ffn_fold(const float *logits, const float *mats, const float *banks,
                const float *combine, float *F, int d, int nb, void *stream);

/* Workspace bytes dp_ffn_fwd needs for `tokens` rows of width d. */
DP_API size_t dp_ffn_workspace_size(int tokens, int d, int x_dtype);

/*
 * Spectral Lerp FFN forward: h_b = M_b x via the fast transforms (Sylvester FWHT,
 * the reference's recursive Haar) and one GEMM with the DCT-II matrix,
 * z = [cos h_b, sin h_b]_b, y = z F (F from dp_ffn_fold).
 * Replaces LearnableSubstrateLerpFFN.forward (delta_phase/layers.py:119-141) and the
 * dense bases of delta_phase/spectral.py:4-35.
 *   x, y (tokens, d), dct (d, d) = mat_dct, F (6d, d): all contiguous and of dtype
 *   x_dtype (DP_F32: TF32 tensor-core GEMMs; DP_BF16: bf16 GEMMs), fp32 accumulation.
 *   Both GEMMs run on the library's own tcgen05 kernel for d >= 64 (bf16) or d >= 32
 *   (float32), on a CUDA-core kernel below that; no library GEMM and no handle.
 *   d a power of two, 8 <= d <= 4096.  workspace >= dp_ffn_workspace_size() bytes,
 *   256-byte aligned.
 */
DP_API int dp_ffn_fwd(const void *x, int x_dtype, const void *dct, const void *F, void *y, int tokens,
               int d, void *workspace, size_t workspace_bytes, void *stream);

/*
 * The FFN with the block's residual add: y += FFN(x), y (tokens, d) float32, added in
 * the combine GEMM's epilogue.  The block output x + ffn(norm2(x)) of
 * DeltaPhaseHolographicBlock.forward/step (delta_phase/layers.py:243, 290) and of
 * ComplexBetaDeltaPhaseBlock (layers.py:368, 417) with y holding the residual stream.
 * Other arguments and limits as dp_ffn_fwd (same workspace size).
 */
DP_API int dp_ffn_fwd_residual(const void *x, int x_dtype, const void *dct, const void *F, float *y,
               int tokens, int d, void *workspace, size_t workspace_bytes, void *stream);

/*
 * The middle step of dp_ffn_fwd on its own: z (tokens, 6d) = [cos h_b, sin h_b] for the
 * three branches of LearnableSubstrateLerpFFN.forward (delta_phase/layers.py:119-141),
 * FWHT and Haar from x, the DCT branch from its projections hdct = x mat_dct^T
 * (tokens, d) float32.  x and z of dtype x_dtype (float32 or bf16), contiguous; hdct
 * and z 16-byte aligned.  Lets a caller run the two GEMMs around it with its own GEMM
 * (dp_gemm_skinny for decode batches).
 */
DP_API int dp_ffn_features(const void *x, int x_dtype, const float *hdct, void *z, int tokens, int d,
               void *stream);

/*
 * Skinny GEMM for decode batches: y (M, N) = x (M, K) W^T (+ bias) (+ y if accumulate),
 * the token-step projections of the blocks (delta_phase/layers.py:262-290; nn.Linear with
 * M = batch rows) and the FFN's two matrix products.
 *   x (M, K) bf16, row stride ldx (a multiple of 8); W (N, K) bf16, contiguous
 *   (nn.Linear weight layout); both 16-byte aligned.  bias (N) of bias_dtype or NULL.
 *   y (M, N) of y_dtype, row stride ldy.  1 <= M <= 16; K a multiple of 32.
 * fp32 accumulation; deterministic (the K split is summed in a fixed order).
 */
DP_API int dp_gemm_skinny(const void *x, int64_t ldx, const void *w, const void *bias, int bias_dtype,
               void *y, int y_dtype, int64_t ldy, int accumulate, int M, int N, int K, void *stream);

/*
 * Allocation-free variant of dp_ffn_fwd.  It has no counterpart in the reference.
 * For callers that cannot allocate device memory where they run the FFN: code being
 * captured into a CUDA graph (cudaMalloc cannot be captured), runtimes whose own
 * allocator owns the device heap, and decode loops that must not block on the
 * driver's allocator.  Same arguments and results as dp_ffn_fwd, but no workspace: the
 * scratch is a fixed 8 MiB array in the library's device image (held on every GPU that
 * loads the library until exit), and the GEMMs run on CUDA cores (the tensor-core path
 * of dp_ffn_fwd keeps F^T in its workspace).
 * Limit: tokens <= dp_ffn_noalloc_max_tokens(d, x_dtype) (511 at d = 1024 with bf16 x);
 * larger calls fail with DP_ERR_WORKSPACE.  Every call looks up the array's device
 * address (cudaGetSymbolAddress, no allocation); the first call on a device also loads the
 * kernels of both dtypes (CUDA's lazy loading would otherwise load them on first launch),
 * so make that first call before any stream capture.  Calls share the array and it keeps
 * the last call's contents: calls that overlap on the GPU race and must be serialised.
 */
DP_API int dp_ffn_fwd_noalloc(const void *x, int x_dtype, const void *dct, const void *F, void *y,
                              int tokens, int d, void *stream);
/* Largest token count dp_ffn_fwd_noalloc accepts for width d and dtype x_dtype. */
DP_API size_t dp_ffn_noalloc_max_tokens(int d, int x_dtype);

/*
 * Fused block glue: norm1 and ShortCausalConv1D.forward of DeltaPhaseHolographicBlock
 * (delta_phase/layers.py:60-88,178):  n = LayerNorm(x) (weight ln_w, bias ln_b, eps);
 * out = n + SiLU(b + sum_j w[c][j] n[t - (k-1) + j][c])  (zero before the sequence start).
 *   x, out : (B, L, d) contiguous, float32 or bfloat16 (dtype codes)
 *   conv_w : (d, k) float32 (the depthwise Conv1d weight (d, 1, k));  conv_b : (d) or NULL
 * Limits: k <= 8; (16 + k - 1) * d * 4 bytes of shared memory at most 227 KB.
 */
DP_API int dp_ln_conv_silu(const void *x, int x_dtype, const float *ln_w, const float *ln_b, float eps,
                           const float *conv_w, const float *conv_b, void *out, int out_dtype, int B, int L,
                           int d, int k, void *stream);

/*
 * Decode step of the same (ShortCausalConv1D.step, delta_phase/layers.py:43-50,182-190):
 * n = LayerNorm(x_t); out = n + SiLU(b + sum_{j<k-1} w[c][j] state[c][j] + w[c][k-1] n[c]);
 * then state (B, d, k-1) float32, the conv's last k-1 inputs, shifts left and takes n.
 *   x, out : (B, d) contiguous, float32 or bfloat16;  conv_w : (d, k);  conv_b : (d) or NULL
 */
DP_API int dp_ln_conv_step(const void *x, int x_dtype, const float *ln_w, const float *ln_b, float eps,
                           const float *conv_w, const float *conv_b, float *conv_state, void *out,
                           int out_dtype, int B, int d, int k, void *stream);

/*
 * s = x (+ residual); y = LayerNorm(s) over the last dimension (weight ln_w, bias ln_b, eps).
 * The block's norm_retrieved and norm2 (delta_phase/layers.py:237-243), with the residual
 * add of the output projection fused in front of norm2.
 *   x : (rows, d) float32 or bfloat16;  residual, sum_out : (rows, d) float32 or NULL
 *   y : (rows, d) float32 or bfloat16 (y_dtype)
 */
DP_API int dp_layernorm(const void *x, int x_dtype, const float *residual, const float *ln_w,
                        const float *ln_b, float eps, float *sum_out, void *y, int y_dtype, int64_t rows,
                        int d, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* DELTAPHASE_B200_H */
