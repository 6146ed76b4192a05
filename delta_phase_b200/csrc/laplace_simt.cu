// LaplacePhaseCore chunkwise forward (gated per-row decay), CUDA cores, fp32.
//
// Reference: LaplacePhaseCore.forward (delta_phase/layers.py:481-561), token-loop
// oracle forward_sequential (layers.py:563-583), mcarbonell/delta-phase v1.3.0.
//
// Recurrence per (batch, head):  v_old = S kap_t / D  (pre-decay state);
//   S = diag(r_t) S + beta_t (v_t - v_old) kap_t^T;  out_t = S xi_t / D,
// with kap_t = e^{sigma_k} [cos th, sin th] interleaved, r_t = exp(max(log r_t, -80))
// (the reference clamps each step's log-decay at LOG_FLOOR = -80, layers.py:445,512).
// Within a chunk, with the in-chunk cumulative log-decay Lc[m, o] (Lc[-1] = 0):
//   e_m[o] = v_m[o] - exp(Lc[m-1,o]) (S0 kap_m)[o]/D
//            - sum_{s<m} exp(Lc[m-1,o] - Lc[s,o]) beta_s g[s,m] e_s[o]     (g = kap_s.kap_m/D)
//   out_m[o] = exp(Lc[m,o]) (S0 xi_m)[o]/D + sum_{s<=m} exp(Lc[m,o] - Lc[s,o]) beta_s e_s[o] h[s,m]
//   S[o,:]  = exp(Lc[C-1,o]) S0[o,:] + sum_s exp(Lc[C-1,o] - Lc[s,o]) beta_s e_s[o] kap_s
// This is the reference's per-channel lower-triangular system (layers.py:522-534) with
// every decay ratio formed as exp(difference) -- always <= 1 -- instead of the
// reference's exp(-Lc) factorisation (layers.py:540), which overflows once a chunk's
// cumulative log-decay passes -88.  Tokens past L behave as the reference's padding
// (r = 1, beta = 0).
#include "dp_common.cuh"

namespace dp {
namespace {

constexpr int kLapThreads = 256;
constexpr float kLogFloor = -80.0f;

__device__ __forceinline__ float load_any(const void *p, int dt, int64_t i) {
  if (dt == DP_F32) return static_cast<const float *>(p)[i];
  if (dt == DP_BF16) return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
  return __half2float(static_cast<const __half *>(p)[i]);
}

__host__ __device__ inline size_t lap_smem_floats(int CI, int D, int Dv) {
  const int ks = 2 * D + 1;
  // S, kap, xi, {v->E, B0k, B0q, Lc}, {g, h}, beta
  return (size_t)Dv * ks + 2 * (size_t)CI * ks + 4 * (size_t)CI * (Dv + 1) + 2 * (size_t)CI * CI + CI;
}

struct LapPtrs {
  const void *tk, *mk, *tq, *mq, *v, *lr, *beta;
};

struct LapStrides {  // theta_k, logmag_k, theta_q, logmag_q, v, log_decay, beta, out
  SeqStrides s[8];
};

template <int CI>
__global__ void __launch_bounds__(kLapThreads)
laplace_simt_kernel(LapPtrs p, int in_dt, int beta_dt, const float *state_in, float *out,
                    float *state_out, int H, int L, int D, int Dv, LapStrides sp) {
  extern __shared__ float smem[];
  const int D2 = 2 * D, ks = D2 + 1, vs = Dv + 1;
  float *S = smem;               // Dv x ks
  float *kap = S + Dv * ks;      // CI x ks
  float *xi = kap + CI * ks;     // CI x ks
  float *E = xi + CI * ks;       // CI x vs   v, then e
  float *B0k = E + CI * vs;      // CI x vs
  float *B0q = B0k + CI * vs;    // CI x vs
  float *Lc = B0q + CI * vs;     // CI x vs   cumulative log-decay
  float *g = Lc + CI * vs;       // CI x CI   g[s*CI+m] = kap_s.kap_m / D
  float *hq = g + CI * CI;       // CI x CI   h[s*CI+m] = kap_s.xi_m / D
  float *bb = hq + CI * CI;      // CI

  const SeqStrides s_tk = sp.s[0], s_mk = sp.s[1], s_tq = sp.s[2], s_mq = sp.s[3], s_v = sp.s[4],
                   s_lr = sp.s[5], s_b = sp.s[6], s_out = sp.s[7];
  const int tid = threadIdx.x, bh = blockIdx.x, b = bh / H, h = bh % H;
  const float inv_d = 1.0f / (float)D;
  const int64_t st_off = (int64_t)bh * Dv * D2;
  for (int idx = tid; idx < Dv * D2; idx += kLapThreads)
    S[(idx / D2) * ks + idx % D2] = state_in ? state_in[st_off + idx] : 0.0f;

  for (int t0 = 0; t0 < L; t0 += CI) {
    __syncthreads();
    for (int idx = tid; idx < CI * D; idx += kLapThreads) {
      const int t = idx / D, c = idx % D, tok = t0 + t;
      float ck = 0.f, sk = 0.f, cq = 0.f, sq = 0.f;
      if (tok < L) {
        const float th_k = load_any(p.tk, in_dt, b * s_tk.b + h * s_tk.h + tok * s_tk.t + c);
        const float th_q = load_any(p.tq, in_dt, b * s_tq.b + h * s_tq.h + tok * s_tq.t + c);
        const float ak = p.mk ? expf(load_any(p.mk, in_dt, b * s_mk.b + h * s_mk.h + tok * s_mk.t + c)) : 1.f;
        const float aq = p.mq ? expf(load_any(p.mq, in_dt, b * s_mq.b + h * s_mq.h + tok * s_mq.t + c)) : 1.f;
        sincosf(th_k, &sk, &ck);
        sincosf(th_q, &sq, &cq);
        ck *= ak; sk *= ak; cq *= aq; sq *= aq;
      }
      kap[t * ks + 2 * c] = ck;
      kap[t * ks + 2 * c + 1] = sk;
      xi[t * ks + 2 * c] = cq;
      xi[t * ks + 2 * c + 1] = sq;
    }
    for (int idx = tid; idx < CI * Dv; idx += kLapThreads) {
      const int t = idx / Dv, o = idx % Dv, tok = t0 + t;
      E[t * vs + o] = tok < L ? load_any(p.v, in_dt, b * s_v.b + h * s_v.h + tok * s_v.t + o) : 0.f;
    }
    for (int t = tid; t < CI; t += kLapThreads)
      bb[t] = (t0 + t < L) ? load_any(p.beta, beta_dt, b * s_b.b + h * s_b.h + (int64_t)(t0 + t) * s_b.t) : 0.f;
    // cumulative clamped log-decay per value channel (one thread per channel)
    for (int o = tid; o < Dv; o += kLapThreads) {
      float acc = 0.f;
      for (int t = 0; t < CI; ++t) {
        const int tok = t0 + t;
        if (tok < L)
          acc += fmaxf(load_any(p.lr, in_dt, b * s_lr.b + h * s_lr.h + tok * s_lr.t + o), kLogFloor);
        Lc[t * vs + o] = acc;
      }
    }
    __syncthreads();

    for (int idx = tid; idx < CI * CI; idx += kLapThreads) {
      const int s = idx / CI, m = idx % CI;
      float gg = 0.f, hh = 0.f;
      if (s <= m) {
        const float *a = kap + s * ks, *bk = kap + m * ks, *bq = xi + m * ks;
        for (int j = 0; j < D2; ++j) {
          gg = fmaf(a[j], bk[j], gg);
          hh = fmaf(a[j], bq[j], hh);
        }
      }
      g[idx] = gg * inv_d;
      hq[idx] = hh * inv_d;
    }
    for (int idx = tid; idx < CI * Dv; idx += kLapThreads) {
      const int m = idx / Dv, o = idx % Dv;
      const float *km = kap + m * ks, *qm = xi + m * ks, *so = S + o * ks;
      float rk = 0.f, rq = 0.f;
      for (int j = 0; j < D2; ++j) {
        rk = fmaf(km[j], so[j], rk);
        rq = fmaf(qm[j], so[j], rq);
      }
      B0k[m * vs + o] = rk * inv_d;
      B0q[m * vs + o] = rq * inv_d;
    }
    __syncthreads();

    // per-channel forward substitution
    if (Dv <= 32) {
      // few channels (small heads): one warp per channel, lane s forms the term of token
      // s < m and a warp sum gives e_m, so the serial depth is CI sums, not CI^2 / 2 terms
      const int lane = tid & 31, warp = tid >> 5;
      for (int o = warp; o < Dv; o += kLapThreads / 32) {
        const float lo = lane < CI ? Lc[lane * vs + o] : 0.f;
        const float bo = lane < CI ? bb[lane] : 0.f;
        float e_lane = 0.f;  // e of token `lane` once solved
        for (int m = 0; m < CI; ++m) {
          const float lprev = m > 0 ? Lc[(m - 1) * vs + o] : 0.f;
          float term = lane < m ? expf(lprev - lo) * bo * g[lane * CI + m] * e_lane : 0.f;
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) term += __shfl_xor_sync(0xffffffffu, term, off);
          const float e = E[m * vs + o] - expf(lprev) * B0k[m * vs + o] - term;
          if (lane == m) e_lane = e;
        }
        if (lane < CI) E[lane * vs + o] = e_lane;
      }
    } else {
      // one thread per value channel
      for (int o = tid; o < Dv; o += kLapThreads) {
        for (int m = 0; m < CI; ++m) {
          const float lprev = m > 0 ? Lc[(m - 1) * vs + o] : 0.f;
          float e = E[m * vs + o] - expf(lprev) * B0k[m * vs + o];
          for (int s = 0; s < m; ++s)
            e -= expf(lprev - Lc[s * vs + o]) * bb[s] * g[s * CI + m] * E[s * vs + o];
          E[m * vs + o] = e;
        }
      }
    }
    __syncthreads();

    for (int idx = tid; idx < CI * Dv; idx += kLapThreads) {
      const int m = idx / Dv, o = idx % Dv;
      if (t0 + m < L) {
        const float lm = Lc[m * vs + o];
        float acc = expf(lm) * B0q[m * vs + o];
        for (int s = 0; s <= m; ++s)
          acc += expf(lm - Lc[s * vs + o]) * bb[s] * E[s * vs + o] * hq[s * CI + m];
        float *op = out + b * s_out.b + h * s_out.h + (int64_t)(t0 + m) * s_out.t + o;
        *op = acc;
      }
    }
    // state carry:  w[s][o] = exp(Lc[C-1] - Lc[s]) beta_s e_s  (stored into B0k)
    __syncthreads();
    for (int idx = tid; idx < CI * Dv; idx += kLapThreads) {
      const int s = idx / Dv, o = idx % Dv;
      B0k[s * vs + o] = expf(Lc[(CI - 1) * vs + o] - Lc[s * vs + o]) * bb[s] * E[s * vs + o];
    }
    __syncthreads();
    for (int idx = tid; idx < Dv * D2; idx += kLapThreads) {
      const int o = idx / D2, j = idx % D2;
      float acc = expf(Lc[(CI - 1) * vs + o]) * S[o * ks + j];
      for (int s = 0; s < CI; ++s) acc = fmaf(B0k[s * vs + o], kap[s * ks + j], acc);
      S[o * ks + j] = acc;
    }
  }
  __syncthreads();
  for (int idx = tid; idx < Dv * D2; idx += kLapThreads)
    state_out[st_off + idx] = S[(idx / D2) * ks + idx % D2];
}

}  // namespace

bool laplace_tc_supported(const void *const *ptrs, int in_dt, const float *out, int D, int Dv,
                          const SeqStrides *s);
int laplace_fwd_tc(const void *const *ptrs, const void *beta, int beta_dt, const float *state_in, float *out,
                   float *state_out, int B, int H, int L, const SeqStrides *s, cudaStream_t stream);

}  // namespace dp

extern "C" int dp_laplace_fwd(const void *theta_k, const void *logmag_k, const void *theta_q,
                              const void *logmag_q, const void *v, const void *log_decay,
                              const void *beta, int in_dtype, int beta_dtype,
                              const float *state_in, float *out, float *state_out, int B, int H,
                              int L, int D, int Dv, int chunk_size, const int64_t *strides,
                              void *stream) {
  using namespace dp;
  DP_REQUIRE(B >= 0 && H >= 0 && L >= 0 && D >= 1 && Dv >= 1 && chunk_size >= 1,
             DP_ERR_INVALID_ARGUMENT, "dp_laplace_fwd: bad sizes");
  DP_REQUIRE(D <= 128 && Dv <= 128, DP_ERR_UNSUPPORTED, "dp_laplace_fwd: D and Dv must be <= 128");
  DP_REQUIRE(valid_dtype(in_dtype) && valid_dtype(beta_dtype), DP_ERR_INVALID_ARGUMENT,
             "dp_laplace_fwd: bad dtype code");
  if (B == 0 || H == 0) return DP_OK;
  DP_REQUIRE(state_out && strides, DP_ERR_INVALID_ARGUMENT, "dp_laplace_fwd: null state_out/strides");
  DP_REQUIRE(L == 0 || (theta_k && theta_q && v && log_decay && beta && out),
             DP_ERR_INVALID_ARGUMENT, "dp_laplace_fwd: null input pointer");
  LapStrides st;
  for (int i = 0; i < 8; ++i) st.s[i] = SeqStrides{strides[3 * i], strides[3 * i + 1], strides[3 * i + 2]};
  LapPtrs p{theta_k, logmag_k, theta_q, logmag_q, v, log_decay, beta};
  if (L > 0) {
    const void *tc_ptrs[6] = {theta_k, logmag_k, theta_q, logmag_q, v, log_decay};
    if (laplace_tc_supported(tc_ptrs, in_dtype, out, D, Dv, st.s))
      return laplace_fwd_tc(tc_ptrs, beta, beta_dtype, state_in, out, state_out, B, H, L, st.s,
                            as_stream(stream));
  }
  const bool ci32 = lap_smem_floats(32, D, Dv) * sizeof(float) <= 200 * 1024;
  const size_t smem = lap_smem_floats(ci32 ? 32 : 16, D, Dv) * sizeof(float);
  DP_REQUIRE(smem <= 227 * 1024, DP_ERR_UNSUPPORTED, "dp_laplace_fwd: shape exceeds shared memory");
  auto kern = ci32 ? laplace_simt_kernel<32> : laplace_simt_kernel<16>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return set_error(DP_ERR_CUDA, std::string("laplace smem attr: ") + cudaGetErrorString(e));
  kern<<<B * H, kLapThreads, smem, as_stream(stream)>>>(p, in_dtype, beta_dtype, state_in, out,
                                                        state_out, H, L, D, Dv, st);
  return check_launch("laplace_simt_kernel");
}
