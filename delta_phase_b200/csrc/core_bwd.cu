// Backward of the complex delta rule (training path): gradients of the chunkwise core
// with respect to theta_k, theta_q, v, beta (or phi of the complex beta) and the initial
// state, given the gradients of the outputs and of the final state.
//
// The reference trains through PyTorch autograd of its chunkwise path
// (_chunkwise_delta_reference, delta_phase/kernels/triton_chunk_delta.py:211-252, via the
// dispatcher at :279-291; DeltaPhaseTritonFunction.backward at :271-276 raises) and of the
// complex-beta token loop (delta_phase/layers.py:346-360).  Both compute the token
// recurrence, per value row o (real form, see core_simt.cu):
//   e_t = v_t - S_{t-1} kap_t / D,  u_t = g_t e_t,  S_t = S_{t-1} + u_t w_t^T,
//   o_t = S_t xi_t / D
// with g = beta, w = kap (real beta) or g = 1, w = beta kap = (br c - bi s, br s + bi c)
// (complex beta, br = 1 + cos phi, bi = sin phi).  Its adjoint, backwards in t with
// dS = dL/dS_t:
//   dS += dO_t xi_t^T / D;  dxi_t = S_t^T dO_t / D;  du_t = dS w_t;  dw_t = dS^T u_t;
//   dg_t = du_t . e_t;  de_t = g_t du_t = dv_t;  S_{t-1} = S_t - u_t w_t^T;
//   dS -= de_t kap_t^T / D;  dkap_t = -S_{t-1}^T de_t / D (+ dw_t through w),
// and dtheta = -sin dkap_cos + cos dkap_sin.  The states S_{t-1} are not stored: the
// kernel runs the recurrence forward once (fp32, keeping u_t in the workspace) and then
// undoes one rank-1 update per token on the way back, which is exact up to fp32
// rounding (no factor multiplies S, so rounding errors only add).  e_t comes back from
// S_t kap_t = S_{t-1} kap_t + u_t (w_t . kap_t), w . kap = D (real) or br D (complex).
//
// One CTA of 256 threads per (b, h): warp w holds rows 32 (w / 4) .. +31 of column
// 32 (w % 4) + lane of S and dS in registers (D <= 64, Dv <= 64).  Row sums (S kap,
// dS w) are warp reduce-scatters plus a 4-way shared-memory sum; column sums (the key /
// query gradients) pair the two row halves through shared memory one token later.  One
// block barrier per token.
#include "dp_common.cuh"

namespace dp {
namespace {

constexpr int kBwdThreads = 256;
constexpr int TB = 32;  // tokens staged per block

struct BwdArgs {
  const void *tk, *tq, *v, *g;  // g: beta or phi
  int in_dt, g_dt;
  SeqStrides s_tk, s_tq, s_v, s_g;
  const float *state_in, *dout, *dstate_out;  // dout (B,H,L,Dv) contiguous; others may be null
  float *dtk, *dtq, *dv, *dg, *dstate_in;     // dtk/dtq (B,H,L,D), dv (B,H,L,Dv), dg (B,H,L)
  float *ws_u;                                // (B,H,L,Dv)
  int H, L, D, Dv;
};

struct Stage {
  float tk[TB][64], tq[TB][64];
  float v[TB][64], dout[TB][64], u[TB][64];
  float g[TB];
};

__device__ __forceinline__ float load_any(const void *p, int dt, int64_t i) {
  if (dt == DP_F32) return static_cast<const float *>(p)[i];
  if (dt == DP_BF16) return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
  return __half2float(static_cast<const __half *>(p)[i]);
}

// Lane l returns the sum over the warp's lanes of x[l] (reduce-scatter of 32 values).
__device__ __forceinline__ float warp_reduce_scatter32(float (&x)[32], int lane) {
#pragma unroll
  for (int k = 16; k >= 1; k >>= 1) {
    const bool upper = (lane & k) != 0;
#pragma unroll
    for (int i = 0; i < k; ++i) {
      const float send = upper ? x[i] : x[i + k];
      const float keep = upper ? x[i + k] : x[i];
      x[i] = keep + __shfl_xor_sync(0xffffffffu, send, k);
    }
  }
  return x[0];
}

// Stages tokens [t0, t0 + n) of this (b, h): phases, values (and output gradients and
// u_t in the backward pass), the write gate.  Rows / channels past Dv / D are zero.
__device__ void stage_tokens(const BwdArgs &a, Stage &st, int b, int h, int t0, int n, bool bwd, int64_t row_base) {
  const int tid = threadIdx.x;
  for (int idx = tid; idx < TB * 64; idx += kBwdThreads) {
    const int r = idx >> 6, c = idx & 63, t = t0 + r;
    const bool ok = r < n;
    float xk = 0.f, xq = 0.f, xv = 0.f, xo = 0.f, xu = 0.f;
    if (ok && c < a.D) {
      xk = load_any(a.tk, a.in_dt, b * a.s_tk.b + h * a.s_tk.h + (int64_t)t * a.s_tk.t + c);
      xq = load_any(a.tq, a.in_dt, b * a.s_tq.b + h * a.s_tq.h + (int64_t)t * a.s_tq.t + c);
    }
    if (ok && c < a.Dv) {
      xv = load_any(a.v, a.in_dt, b * a.s_v.b + h * a.s_v.h + (int64_t)t * a.s_v.t + c);
      if (bwd) {
        xo = a.dout[row_base + (int64_t)t * a.Dv + c];
        xu = a.ws_u[row_base + (int64_t)t * a.Dv + c];
      }
    }
    st.tk[r][c] = xk;
    st.tq[r][c] = xq;
    st.v[r][c] = xv;
    st.dout[r][c] = xo;
    st.u[r][c] = xu;
  }
  for (int r = tid; r < TB; r += kBwdThreads)
    st.g[r] = r < n ? load_any(a.g, a.g_dt, b * a.s_g.b + h * a.s_g.h + (int64_t)(t0 + r) * a.s_g.t) : 0.f;
}

// Column sums of one token -> d theta_k, d theta_q (and d phi).  Called by whole warps
// (the four column warps of row half 0); lane pairs (2c, 2c + 1) hold channel c.
// pend = {sin, cos of theta_k, sin, cos of theta_q, br, bi} of that token.
template <bool CB>
__device__ __forceinline__ void finish_token(const BwdArgs &a, const float (*cb_)[3][128], int j, int lane,
                                             bool col_ok, int64_t gi_base, int t, const float (&pend)[6],
                                             float invD) {
  const float qk = cb_[0][0][j] + cb_[1][0][j];  // d kap through the read (per column)
  const float qq = cb_[0][1][j] + cb_[1][1][j];  // D * d xi
  const float qw = cb_[0][2][j] + cb_[1][2][j];  // d w
  const float ok_ = __shfl_xor_sync(0xffffffffu, qk, 1), oq = __shfl_xor_sync(0xffffffffu, qq, 1),
              ow = __shfl_xor_sync(0xffffffffu, qw, 1);
  const float sk = pend[0], ck = pend[1], sq = pend[2], cq = pend[3], br = pend[4], bi = pend[5];
  float dphi = 0.f;
  if (!(j & 1) && col_ok) {  // even lane: channel j / 2, own = cos column, partner = sin column
    float dkc = qk, dks = ok_;
    if (CB) {
      dkc += br * qw + bi * ow;
      dks += -bi * qw + br * ow;
      const float dbr = -bi, dbi = br - 1.f;
      dphi = qw * (dbr * ck - dbi * sk) + ow * (dbr * sk + dbi * ck);
    } else {
      dkc += qw;
      dks += ow;
    }
    const int64_t gi = gi_base + (j >> 1);
    a.dtk[gi] = -sk * dkc + ck * dks;
    a.dtq[gi] = (-sq * qq + cq * oq) * invD;
  }
  if (CB) {
#pragma unroll
    for (int o2 = 1; o2 < 32; o2 <<= 1) dphi += __shfl_xor_sync(0xffffffffu, dphi, o2);
    if (lane == 0) atomicAdd(&a.dg[t], dphi);
  }
}

template <bool CB>
__global__ void __launch_bounds__(kBwdThreads, 1) core_bwd_kernel(BwdArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  Stage &st = *reinterpret_cast<Stage *>(smem_raw);
  float(*red)[2][4][64] = reinterpret_cast<float(*)[2][4][64]>(smem_raw + sizeof(Stage));  // [parity][which][cb][row]
  float(*colb)[2][3][128] =
      reinterpret_cast<float(*)[2][3][128]>(smem_raw + sizeof(Stage) + sizeof(float) * 2 * 2 * 4 * 64);  // [par][rh][q][j]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rh = warp >> 2, cb = warp & 3, j = 32 * cb + lane, row0 = 32 * rh;
  const int bh = blockIdx.x, b = bh / a.H, h = bh % a.H;
  const int L = a.L, D = a.D, Dv = a.Dv, c_idx = j >> 1;
  const bool col_ok = j < 2 * D;
  const float invD = 1.0f / (float)D;
  const int64_t row_base = (int64_t)bh * L * Dv;  // (B,H,L,Dv) contiguous
  const int64_t st_base = (int64_t)bh * Dv * 2 * D;

  float S[32], dS[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int o = row0 + i;
    S[i] = (a.state_in && col_ok && o < Dv) ? a.state_in[st_base + (int64_t)o * 2 * D + j] : 0.f;
  }

  // ---- pass 1: the recurrence forward, u_t to the workspace
  int par = 0;
  for (int t0 = 0; t0 < L; t0 += TB) {
    const int n = min(TB, L - t0);
    __syncthreads();
    stage_tokens(a, st, b, h, t0, n, false, row_base);
    __syncthreads();
    for (int r = 0; r < n; ++r, par ^= 1) {
      float sk, ck;
      __sincosf(st.tk[r][c_idx & 63], &sk, &ck);
      const float kap = col_ok ? ((j & 1) ? sk : ck) : 0.f;
      float wj = kap;
      const float g = st.g[r];
      float br = 1.f, bi = 0.f;
      if (CB) {
        float sp, cp;
        __sincosf(g, &sp, &cp);
        br = 1.f + cp;
        bi = sp;
        wj = col_ok ? ((j & 1) ? fmaf(br, sk, bi * ck) : fmaf(br, ck, -bi * sk)) : 0.f;
      }
      float x[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) x[i] = S[i] * kap;
      const float part = warp_reduce_scatter32(x, lane);
      red[par][0][cb][row0 + lane] = part;
      __syncthreads();
      const int o = row0 + lane;
      const float sk_row = red[par][0][0][o] + red[par][0][1][o] + red[par][0][2][o] + red[par][0][3][o];
      const float e = st.v[r][o & 63] - sk_row * invD;
      const float u = CB ? e : g * e;
      if (cb == 0 && o < Dv) a.ws_u[row_base + (int64_t)(t0 + r) * Dv + o] = u;
#pragma unroll
      for (int i = 0; i < 32; ++i) S[i] = fmaf(__shfl_sync(0xffffffffu, u, i), wj, S[i]);
    }
  }

  // ---- pass 2: backwards in t
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int o = row0 + i;
    dS[i] = (a.dstate_out && col_ok && o < Dv) ? a.dstate_out[st_base + (int64_t)o * 2 * D + j] : 0.f;
  }
  __syncthreads();  // pass 1's reads of the stage are done
  int pend_t = -1;  // token whose column sums wait in colb[pend_par]
  int pend_par = 0;
  float pend[6] = {0.f, 1.f, 0.f, 1.f, 1.f, 0.f};
  const int nblk = (L + TB - 1) / TB;
  for (int blk = nblk - 1; blk >= 0; --blk) {
    const int t0 = blk * TB, n = min(TB, L - t0);
    __syncthreads();
    stage_tokens(a, st, b, h, t0, n, true, row_base);
    __syncthreads();
    for (int r = n - 1; r >= 0; --r, par ^= 1) {
      const int t = t0 + r;
      float sk, ck, sq, cq;
      __sincosf(st.tk[r][c_idx & 63], &sk, &ck);
      __sincosf(st.tq[r][c_idx & 63], &sq, &cq);
      const float kap = col_ok ? ((j & 1) ? sk : ck) : 0.f;
      const float xi = col_ok ? ((j & 1) ? sq : cq) : 0.f;
      const float g = st.g[r];
      float br = 1.f, bi = 0.f, wj = kap;
      if (CB) {
        float sp, cp;
        __sincosf(g, &sp, &cp);
        br = 1.f + cp;
        bi = sp;
        wj = col_ok ? ((j & 1) ? fmaf(br, sk, bi * ck) : fmaf(br, ck, -bi * sk)) : 0.f;
      }
      // A1: output term, column partials, row products
      float pq = 0.f, pw = 0.f, x1[32], x2[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float dO = st.dout[r][row0 + i];
        const float uu = st.u[r][row0 + i];
        dS[i] = fmaf(dO * invD, xi, dS[i]);
        pq = fmaf(S[i], dO, pq);
        pw = fmaf(dS[i], uu, pw);
        x1[i] = dS[i] * wj;
        x2[i] = S[i] * kap;
      }
      red[par][0][cb][row0 + lane] = warp_reduce_scatter32(x1, lane);
      red[par][1][cb][row0 + lane] = warp_reduce_scatter32(x2, lane);
      __syncthreads();
      // the previous (later) token's column sums: both row halves are in colb now
      if (pend_t >= 0 && rh == 0)
        finish_token<CB>(a, colb[pend_par], j, lane, col_ok, (int64_t)bh * L * D + (int64_t)pend_t * D,
                         bh * L + pend_t, pend, invD);
      // A2: row sums -> du, e; dg, dv
      const int o = row0 + lane;
      const float du = red[par][0][0][o] + red[par][0][1][o] + red[par][0][2][o] + red[par][0][3][o];
      const float skr = red[par][1][0][o] + red[par][1][1][o] + red[par][1][2][o] + red[par][1][3][o];
      const float u_o = st.u[r][o & 63];
      const float wk = CB ? br * (float)D : (float)D;  // w . kap
      const float e = st.v[r][o & 63] - (skr - u_o * wk) * invD;
      const float de = CB ? du : g * du;
      if (cb == 0 && o < Dv) a.dv[row_base + (int64_t)t * Dv + o] = de;
      if (!CB && cb == 0) {
        float p = (o < Dv) ? du * e : 0.f;
#pragma unroll
        for (int o2 = 16; o2 >= 1; o2 >>= 1) p += __shfl_xor_sync(0xffffffffu, p, o2);
        if (lane == 0) atomicAdd(&a.dg[(int64_t)bh * L + t], p);
      }
      // A3: undo the update, propagate dS, read-key partial
      float pk = 0.f;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float de_i = __shfl_sync(0xffffffffu, de, i);
        const float uu = st.u[r][row0 + i];
        S[i] = fmaf(-uu, wj, S[i]);
        dS[i] = fmaf(-de_i * invD, kap, dS[i]);
        pk = fmaf(S[i], de_i, pk);
      }
      colb[par][rh][0][j] = -pk * invD;
      colb[par][rh][1][j] = pq;
      colb[par][rh][2][j] = pw;
      pend_t = t;
      pend_par = par;
      pend[0] = sk;
      pend[1] = ck;
      pend[2] = sq;
      pend[3] = cq;
      pend[4] = br;
      pend[5] = bi;
    }
  }
  __syncthreads();
  if (pend_t >= 0 && rh == 0)
    finish_token<CB>(a, colb[pend_par], j, lane, col_ok, (int64_t)bh * L * D + (int64_t)pend_t * D, bh * L + pend_t,
                     pend, invD);
  if (a.dstate_in) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int o = row0 + i;
      if (col_ok && o < Dv) a.dstate_in[st_base + (int64_t)o * 2 * D + j] = dS[i];
    }
  }
}

}  // namespace
}  // namespace dp

extern "C" size_t dp_core_bwd_workspace_size(int B, int H, int L, int Dv) {
  if (B <= 0 || H <= 0 || L <= 0 || Dv <= 0) return 0;
  return (size_t)B * H * L * Dv * sizeof(float);
}

extern "C" int dp_core_bwd(const void *theta_k, const void *theta_q, const void *v, const void *beta,
                           int in_dtype, int beta_dtype, int complex_beta, const float *state_in,
                           const float *grad_out, const float *grad_state_out, float *grad_theta_k,
                           float *grad_theta_q, float *grad_v, float *grad_beta, float *grad_state_in,
                           int B, int H, int L, int D, int Dv, const int64_t *strides, void *workspace,
                           size_t workspace_bytes, void *stream) {
  using namespace dp;
  DP_REQUIRE(B >= 0 && H >= 0 && L >= 0, DP_ERR_INVALID_ARGUMENT, "dp_core_bwd: negative size");
  DP_REQUIRE(D >= 1 && Dv >= 1, DP_ERR_INVALID_ARGUMENT, "dp_core_bwd: D and Dv must be >= 1");
  DP_REQUIRE(D <= 64 && Dv <= 64, DP_ERR_UNSUPPORTED, "dp_core_bwd: D and Dv must be <= 64");
  DP_REQUIRE(valid_dtype(in_dtype) && valid_dtype(beta_dtype), DP_ERR_INVALID_ARGUMENT, "dp_core_bwd: bad dtype code");
  if (B == 0 || H == 0) return DP_OK;
  DP_REQUIRE(strides, DP_ERR_INVALID_ARGUMENT, "dp_core_bwd: null strides");
  if (L > 0) {
    DP_REQUIRE(theta_k && theta_q && v && beta && grad_out && grad_theta_k && grad_theta_q && grad_v && grad_beta,
               DP_ERR_INVALID_ARGUMENT, "dp_core_bwd: null pointer");
    DP_REQUIRE(workspace && workspace_bytes >= dp_core_bwd_workspace_size(B, H, L, Dv), DP_ERR_WORKSPACE,
               "dp_core_bwd: workspace too small (dp_core_bwd_workspace_size)");
  }
  cudaStream_t s = as_stream(stream);
  if (L > 0) {
    // beta / phi gradients are accumulated with atomics
    cudaError_t e = cudaMemsetAsync(grad_beta, 0, (size_t)B * H * L * sizeof(float), s);
    if (e != cudaSuccess) return set_error(DP_ERR_CUDA, std::string("dp_core_bwd: memset: ") + cudaGetErrorString(e));
  }
  BwdArgs a;
  a.tk = theta_k;
  a.tq = theta_q;
  a.v = v;
  a.g = beta;
  a.in_dt = in_dtype;
  a.g_dt = beta_dtype;
  a.s_tk = SeqStrides{strides[0], strides[1], strides[2]};
  a.s_tq = SeqStrides{strides[3], strides[4], strides[5]};
  a.s_v = SeqStrides{strides[6], strides[7], strides[8]};
  a.s_g = SeqStrides{strides[9], strides[10], strides[11]};
  a.state_in = state_in;
  a.dout = grad_out;
  a.dstate_out = grad_state_out;
  a.dtk = grad_theta_k;
  a.dtq = grad_theta_q;
  a.dv = grad_v;
  a.dg = grad_beta;
  a.dstate_in = grad_state_in;
  a.ws_u = static_cast<float *>(workspace);
  a.H = H;
  a.L = L;
  a.D = D;
  a.Dv = Dv;
  const size_t smem = sizeof(Stage) + sizeof(float) * (2 * 2 * 4 * 64 + 2 * 2 * 3 * 128);
  auto kern = complex_beta ? core_bwd_kernel<true> : core_bwd_kernel<false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return set_error(DP_ERR_CUDA, std::string("dp_core_bwd smem attr: ") + cudaGetErrorString(e));
  kern<<<B * H, kBwdThreads, smem, s>>>(a);
  return check_launch("core_bwd_kernel");
}
