// General-shape chunkwise complex delta-rule forward (CUDA cores, fp32), and the
// phasor Gram kernel.
//
// Reference: _chunkwise_delta_reference (delta_phase/kernels/triton_chunk_delta.py:211-252)
// and gram_matrix_reference (:192-208), mcarbonell/delta-phase v1.3.0.
//
// Real form of the complex rule.  With the key phasor k = e^{i theta} written as the
// interleaved real vector kap = [cos th_0, sin th_0, cos th_1, sin th_1, ...] (2D) and
// the complex state M (Dv x D) as the real matrix S (Dv x 2D) of its interleaved
// (re, im) pairs:  Re(M conj(k)) = S kap,  Re(K K^H) = kap kap^T, and M += u k^T is
// S += u kap^T.  Per chunk of Ci tokens (kap rows K, xi rows Q, values V, beta):
//   A = strict_lower(K K^T / D) diag(beta),  T = (I + A)^-1
//   U = diag(beta) T (V - K S^T / D)
//   O = Q S^T / D + tril(Q K^T / D) U
//   S += U^T K
// which is the reference's chunk step with its beta / transpose conventions
// (lower entry [t, s] of I + L^T is beta_s G[t, s]).  The result does not depend
// on the chunk length, so the kernel uses its own internal chunk Ci.
//
// One CTA per (batch, head); the state lives in shared memory for the whole
// sequence.  This kernel covers every shape (D, Dv <= 128, any L); the tensor-core
// kernel in core_tc.cu covers the (D = Dv = 64) production shape.
//
// Complex beta (ComplexBetaDeltaPhaseBlock, delta_phase/layers.py:294-418; beta_t =
// 1 + e^{i phi_t}, update M += beta (v - Re(M conj k) / D) k^T): in the real form the
// update writes along w_t = beta_t k_t = (br c - bi s, br s + bi c) per channel while
// the read stays along kap_t, so S_t = S_{t-1} + (v_t - S_{t-1} kap_t / D) w_t^T and
//   A = strict_lower(K W^T / D),  T = (I + A)^-1,  U = T (V - K S^T / D)
//   O = Q S^T / D + tril(Q W^T / D) U,  S += U^T W.
#include "dp_common.cuh"

namespace dp {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float load_beta(const void *p, int dt, int64_t i) {
  if (dt == DP_F32) return static_cast<const float *>(p)[i];
  if (dt == DP_BF16) return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
  return __half2float(static_cast<const __half *>(p)[i]);
}

template <int CI>
__host__ __device__ inline size_t core_simt_smem_floats(int D, int Dv, bool cbeta) {
  const int ks = 2 * D + 1;
  return (size_t)Dv * ks + (cbeta ? 3 : 2) * (size_t)CI * ks + 3 * (size_t)CI * Dv + 3 * CI * CI + CI;
}

// CB: `beta` holds phi of the complex beta 1 + e^{i phi}.
template <typename T, int CI, bool CB>
__global__ void __launch_bounds__(kThreads)
core_fwd_simt_kernel(const T *__restrict__ tk, const T *__restrict__ tq, const T *__restrict__ v,
                     const void *__restrict__ beta, int beta_dt, const float *state_in,
                     float *__restrict__ out, float *state_out, int H, int L, int D,
                     int Dv, SeqStrides s_tk, SeqStrides s_tq, SeqStrides s_v, SeqStrides s_b,
                     SeqStrides s_out) {
  extern __shared__ float smem[];
  const int D2 = 2 * D, ks = D2 + 1;
  float *S = smem;              // Dv x ks     state, interleaved (re, im) columns
  float *kap = S + Dv * ks;     // CI x ks     key phasors
  float *xi = kap + CI * ks;    // CI x ks     query phasors
  float *R = xi + CI * ks;      // CI x Dv     V, then V - K S^T / D
  float *U = R + CI * Dv;       // CI x Dv
  float *Oi = U + CI * Dv;      // CI x Dv     Q S^T / D
  float *A = Oi + CI * Dv;      // CI x CI     beta-scaled strictly-lower Gram
  float *Tm = A + CI * CI;      // CI x CI     (I + A)^-1
  float *P = Tm + CI * CI;      // CI x CI     tril(Q K^T) / D
  float *bb = P + CI * CI;      // CI          beta (CB: phi)
  float *wk = bb + CI;          // CI x ks     CB: write keys beta k

  const int tid = threadIdx.x;
  const int bh = blockIdx.x;
  const int b = bh / H, h = bh % H;
  const float inv_d = 1.0f / (float)D;
  const int64_t st_off = (int64_t)bh * Dv * D2;

  for (int idx = tid; idx < Dv * D2; idx += kThreads)
    S[(idx / D2) * ks + idx % D2] = state_in ? state_in[st_off + idx] : 0.0f;

  const T *tk_bh = tk + b * s_tk.b + h * s_tk.h;
  const T *tq_bh = tq + b * s_tq.b + h * s_tq.h;
  const T *v_bh = v + b * s_v.b + h * s_v.h;
  const int64_t b_bh = b * s_b.b + h * s_b.h;
  float *out_bh = out + b * s_out.b + h * s_out.h;

  for (int t0 = 0; t0 < L; t0 += CI) {
    __syncthreads();
    // 1. phasors, values, beta of this chunk (rows past L are zero, beta = 0)
    for (int idx = tid; idx < CI * D; idx += kThreads) {
      const int t = idx / D, c = idx % D, tok = t0 + t;
      float ck = 0.f, sk = 0.f, cq = 0.f, sq = 0.f;
      if (tok < L) {
        phase_sincos(tk_bh[tok * s_tk.t + c], &sk, &ck);
        phase_sincos(tq_bh[tok * s_tq.t + c], &sq, &cq);
      }
      kap[t * ks + 2 * c] = ck;
      kap[t * ks + 2 * c + 1] = sk;
      xi[t * ks + 2 * c] = cq;
      xi[t * ks + 2 * c + 1] = sq;
    }
    for (int idx = tid; idx < CI * Dv; idx += kThreads) {
      const int t = idx / Dv, o = idx % Dv, tok = t0 + t;
      R[idx] = tok < L ? to_f32(v_bh[tok * s_v.t + o]) : 0.f;
    }
    for (int t = tid; t < CI; t += kThreads)
      bb[t] = (t0 + t < L) ? load_beta(beta, beta_dt, b_bh + (int64_t)(t0 + t) * s_b.t) : 0.f;
    __syncthreads();
    if (CB) {
      for (int idx = tid; idx < CI * D; idx += kThreads) {
        const int t = idx / D, c = idx % D;
        float sp, cp;
        sincosf(bb[t], &sp, &cp);
        const float br = 1.f + cp, c0 = kap[t * ks + 2 * c], s0 = kap[t * ks + 2 * c + 1];
        wk[t * ks + 2 * c] = fmaf(br, c0, -sp * s0);
        wk[t * ks + 2 * c + 1] = fmaf(br, s0, sp * c0);
      }
      __syncthreads();
    }
    const float *wsrc = CB ? wk : kap;  // write keys

    // 2. Gram (A), intra-chunk query-key products (P), state reads (R, Oi)
    for (int idx = tid; idx < CI * CI; idx += kThreads) {
      const int t = idx / CI, s = idx % CI;
      float g = 0.f, p = 0.f;
      if (s <= t) {
        const float *kt = kap + t * ks, *ks_ = wsrc + s * ks, *qt = xi + t * ks;
        for (int j = 0; j < D2; ++j) {
          g = fmaf(kt[j], ks_[j], g);
          p = fmaf(qt[j], ks_[j], p);
        }
      }
      A[idx] = (s < t) ? (CB ? 1.f : bb[s]) * g * inv_d : 0.f;
      P[idx] = (s <= t) ? p * inv_d : 0.f;
    }
    for (int idx = tid; idx < CI * Dv; idx += kThreads) {
      const int t = idx / Dv, o = idx % Dv;
      const float *kt = kap + t * ks, *qt = xi + t * ks, *so = S + o * ks;
      float r = 0.f, q = 0.f;
      for (int j = 0; j < D2; ++j) {
        const float sv = so[j];
        r = fmaf(kt[j], sv, r);
        q = fmaf(qt[j], sv, q);
      }
      R[idx] -= r * inv_d;
      Oi[idx] = q * inv_d;
    }
    __syncthreads();

    // 3. T = (I + A)^-1 by forward substitution; thread j owns column j
    if (tid < CI) {
      float col[CI];
#pragma unroll
      for (int i = 0; i < CI; ++i) {
        float acc = (i == tid) ? 1.f : 0.f;
#pragma unroll
        for (int k = 0; k < i; ++k) acc = fmaf(-A[i * CI + k], col[k], acc);
        col[i] = acc;
      }
#pragma unroll
      for (int i = 0; i < CI; ++i) Tm[i * CI + tid] = col[i];
    }
    __syncthreads();

    // 4. U = diag(beta) T R
    for (int idx = tid; idx < CI * Dv; idx += kThreads) {
      const int t = idx / Dv, o = idx % Dv;
      float acc = 0.f;
      for (int s = 0; s <= t; ++s) acc = fmaf(Tm[t * CI + s], R[s * Dv + o], acc);
      U[idx] = CB ? acc : bb[t] * acc;
    }
    __syncthreads();

    // 5. O = Q S^T / D + P U  (written out);  S += U^T K
    for (int idx = tid; idx < CI * Dv; idx += kThreads) {
      const int t = idx / Dv, o = idx % Dv;
      if (t0 + t < L) {
        float acc = Oi[idx];
        for (int s = 0; s <= t; ++s) acc = fmaf(P[t * CI + s], U[s * Dv + o], acc);
        out_bh[(int64_t)(t0 + t) * s_out.t + o] = acc;
      }
    }
    for (int idx = tid; idx < Dv * D2; idx += kThreads) {
      const int o = idx / D2, j = idx % D2;
      float acc = 0.f;
#pragma unroll 4
      for (int t = 0; t < CI; ++t) acc = fmaf(U[t * Dv + o], wsrc[t * ks + j], acc);
      S[o * ks + j] += acc;
    }
  }
  __syncthreads();
  for (int idx = tid; idx < Dv * D2; idx += kThreads)
    state_out[st_off + idx] = S[(idx / D2) * ks + idx % D2];
}

// G[n, m, j] = beta[n, m] sum_d cos(theta_m - theta_j) / D for m > j (row-beta convention
// of gram_matrix_reference, triton_chunk_delta.py:192-208).
template <typename T>
__global__ void __launch_bounds__(kThreads)
gram_kernel(const T *__restrict__ theta, const void *__restrict__ beta, int beta_dt,
            float *__restrict__ out, int C, int D) {
  extern __shared__ float cs[];  // C x (2D + 1)
  const int n = blockIdx.x, D2 = 2 * D, ks = D2 + 1;
  const T *th = theta + (int64_t)n * C * D;
  for (int idx = threadIdx.x; idx < C * D; idx += kThreads) {
    float s, c;
    phase_sincos(th[idx], &s, &c);
    cs[(idx / D) * ks + 2 * (idx % D)] = c;
    cs[(idx / D) * ks + 2 * (idx % D) + 1] = s;
  }
  __syncthreads();
  const float inv_d = 1.0f / (float)D;
  for (int idx = threadIdx.x; idx < C * C; idx += kThreads) {
    const int m = idx / C, j = idx % C;
    float g = 0.f;
    if (m > j) {
      for (int q = 0; q < D2; ++q) g = fmaf(cs[m * ks + q], cs[j * ks + q], g);
      g = g * inv_d * load_beta(beta, beta_dt, (int64_t)n * C + m);
    }
    out[(int64_t)n * C * C + idx] = g;
  }
}

template <int CI>
int launch_core_simt(const void *tk, const void *tq, const void *v, const void *beta, int in_dt,
                     int beta_dt, const float *state_in, float *out, float *state_out, int B,
                     int H, int L, int D, int Dv, const SeqStrides *s, cudaStream_t stream, bool cbeta) {
  const size_t smem = core_simt_smem_floats<CI>(D, Dv, cbeta) * sizeof(float);
  return dispatch_dtype(in_dt, [&](auto tag) -> int {
    using T = decltype(tag);
    auto kern = cbeta ? core_fwd_simt_kernel<T, CI, true> : core_fwd_simt_kernel<T, CI, false>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return set_error(DP_ERR_CUDA, std::string("core_fwd_simt smem attr: ") + cudaGetErrorString(e));
    kern<<<B * H, kThreads, smem, stream>>>(static_cast<const T *>(tk), static_cast<const T *>(tq),
                                            static_cast<const T *>(v), beta, beta_dt, state_in, out,
                                            state_out, H, L, D, Dv, s[0], s[1], s[2], s[3], s[4]);
    return check_launch("core_fwd_simt_kernel");
  });
}

}  // namespace

// Entry used by dp_core_fwd / dp_core_cbeta_fwd for shapes the tensor-core kernel does not cover.
int core_fwd_simt(const void *tk, const void *tq, const void *v, const void *beta, int in_dt,
                  int beta_dt, const float *state_in, float *out, float *state_out, int B, int H,
                  int L, int D, int Dv, const SeqStrides *s, cudaStream_t stream, bool cbeta) {
  const size_t limit = 227 * 1024;
  if (core_simt_smem_floats<32>(D, Dv, cbeta) * sizeof(float) <= limit)
    return launch_core_simt<32>(tk, tq, v, beta, in_dt, beta_dt, state_in, out, state_out, B, H, L, D, Dv, s, stream,
                                cbeta);
  if (core_simt_smem_floats<16>(D, Dv, cbeta) * sizeof(float) <= limit)
    return launch_core_simt<16>(tk, tq, v, beta, in_dt, beta_dt, state_in, out, state_out, B, H, L, D, Dv, s, stream,
                                cbeta);
  return set_error(DP_ERR_UNSUPPORTED, "core_fwd: D/Dv too large for shared memory");
}

}  // namespace dp

extern "C" int dp_gram(const void *theta, const void *beta, int in_dtype, int beta_dtype,
                       float *out, int N, int C, int D, void *stream) {
  using namespace dp;
  DP_REQUIRE(N >= 0 && C >= 0 && D >= 1, DP_ERR_INVALID_ARGUMENT, "dp_gram: bad sizes");
  DP_REQUIRE(valid_dtype(in_dtype) && valid_dtype(beta_dtype), DP_ERR_INVALID_ARGUMENT, "dp_gram: bad dtype");
  DP_REQUIRE(C <= 256 && D <= 256, DP_ERR_UNSUPPORTED, "dp_gram: C and D must be <= 256");
  if (N == 0 || C == 0) return DP_OK;
  DP_REQUIRE(theta && beta && out, DP_ERR_INVALID_ARGUMENT, "dp_gram: null pointer");
  const size_t smem = (size_t)C * (2 * D + 1) * sizeof(float);
  DP_REQUIRE(smem <= 227 * 1024, DP_ERR_UNSUPPORTED, "dp_gram: C * (2D + 1) * 4 bytes exceeds shared memory");
  return dispatch_dtype(in_dtype, [&](auto tag) -> int {
    using T = decltype(tag);
    auto kern = gram_kernel<T>;
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return set_error(DP_ERR_CUDA, std::string("gram smem attr: ") + cudaGetErrorString(e));
    kern<<<N, kThreads, smem, as_stream(stream)>>>(static_cast<const T *>(theta), beta, beta_dtype,
                                                   out, C, D);
    return check_launch("gram_kernel");
  });
}
