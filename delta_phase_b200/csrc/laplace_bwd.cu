// Backward of the LaplacePhaseCore recurrence (training path): gradients with respect to
// theta_k, log|k|, theta_q, log|q|, v, log r (the per-row decay), beta and the initial state.
//
// The reference trains LaplacePhaseCore through PyTorch autograd of its chunk loop
// (delta_phase/layers.py:481-561; its tests check the gradient flow through the solve,
// tests/test_laplace_chunkwise.py).  The recurrence, per value row o (real form,
// kap = |k| [cos theta_k, sin theta_k] interleaved, xi likewise for q):
//   e_t = v_t - S_{t-1} kap_t / D,  S_t = diag(r_t) S_{t-1} + beta_t e_t kap_t^T,
//   o_t = S_t xi_t / D,  r_t = exp(max(log r_t, -80))  (layers.py:512)
// and its adjoint, backwards in t with dS = dL/dS_t:
//   dS += dO_t xi_t^T / D;  dxi_t = S_t^T dO_t / D;  du_t = dS kap_t;  dkap_t = dS^T u_t;
//   dr_t = rowsum(dS o S_{t-1});  dbeta_t = du_t . e_t;  de_t = beta_t du_t = dv_t;
//   dS <- diag(r_t) dS - de_t kap_t^T / D;  dkap_t -= S_{t-1}^T de_t / D;
//   d log r = r dr (0 where the clamp is active), d theta = -kap_s dkap_c + kap_c dkap_s,
//   d log|k| = kap_c dkap_c + kap_s dkap_s (and the same for q).
// A strong decay (r down to e^-80) makes S_{t-1} unrecoverable from S_t, so nothing is
// undone: pass 1 runs the recurrence forward and keeps the state at every 32-token
// sub-chunk start; pass 2 takes the sub-chunks backwards, recomputes the sub-chunk's
// states from its checkpoint into a per-unit scratch (32 KB per token at D = Dv = 64,
// L2-resident) and then walks back through them.
//
// Rows of the state never interact (each value row has its own decay), so one CTA of 256
// threads takes one (b, h) and one half of its value rows (two CTAs per unit when
// Dv > 32): warp w holds rows 32 rh + 16 (w / 4) .. +15 of column 32 (w % 4) + lane of S
// and dS in registers (D <= 64, Dv <= 64; two warps per scheduler); heads with 2 D <= 32
// and Dv <= 32 take a one-warp-per-unit kernel instead (end of this file).  Row sums are warp reduce-scatters plus a 4-way
// shared-memory sum.  The only sums across rows -- the key / query gradients and d beta --
// are outputs: a CTA sums its two row groups in shared memory in a fixed order, and each
// half adds its part into the zeroed outputs (with two halves the two additions onto zero
// commute exactly, so the result does not depend on their order).
#include "dp_common.cuh"

namespace dp {
namespace {

constexpr int kLT = 256;     // threads: 2 row groups x 4 column blocks
constexpr int kRW = 16;      // state rows per warp
constexpr int kLC = 32;      // tokens per sub-chunk
constexpr int kLF = 128;     // key features (2 D) at most
constexpr int kLDv = 64;     // value rows at most
constexpr float kLogFloor = -80.f;

struct LapBwdArgs {
  const void *tk, *mk, *tq, *mq, *v, *ld, *beta;  // mk, mq may be null (unit magnitudes)
  int in_dt, beta_dt;
  SeqStrides s_tk, s_mk, s_tq, s_mq, s_v, s_ld, s_b;
  const float *state_in, *dout, *dstate_out;  // dout (B,H,L,Dv) contiguous; the others may be null
  float *dtk, *dmk, *dtq, *dmq;               // (B,H,L,D)
  float *dv, *dld;                            // (B,H,L,Dv)
  float *dbeta;                               // (B,H,L), accumulated: zeroed by the entry point
  float *dstate_in;                           // may be null
  float *ckpt;                                // (B*H, NSC, Dv, F) states at sub-chunk starts
  float *scratch;                             // (B*H, kLC + 1, Dv, F) states inside a sub-chunk
  int H, L, D, Dv;
  int nhalf;  // CTAs per unit (value-row halves)
};

struct LapStage {
  float kc[kLC][64], ks[kLC][64];  // key features |k| cos, |k| sin per channel
  float qc[kLC][64], qs[kLC][64];
  float v[kLC][64], r[kLC][64], rg[kLC][64];  // rg = r where log r > -80, else 0 (clamp gradient)
  float dout[kLC][64], u[kLC][64], e[kLC][64];
  float beta[kLC];
};

__device__ __forceinline__ float load_any(const void *p, int dt, int64_t i) {
  if (dt == DP_F32) return static_cast<const float *>(p)[i];
  if (dt == DP_BF16) return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
  return __half2float(static_cast<const __half *>(p)[i]);
}

// Lane l returns the sum over the warp's lanes of x[l] (reduce-scatter of 32 values).
__device__ __forceinline__ float reduce_scatter32(float (&x)[32], int lane) {
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

// Lane l returns the warp sum of x[l % ROWS] (ROWS = 16 or 32).
template <int ROWS>
__device__ __forceinline__ float rs_rows(float (&x)[ROWS], int lane) {
  if (ROWS == 16) {
#pragma unroll
    for (int i = 0; i < 16; ++i) x[i] += __shfl_xor_sync(0xffffffffu, x[i], 16);
  }
#pragma unroll
  for (int k = ROWS / 2; k >= 1; k >>= 1) {
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

// Tokens [t0, t0 + n) of this (b, h) into the stage; every global load of a thread is
// issued before its arithmetic and shared stores.  Rows / channels past n, D, Dv are zero
// (decay 1 for the absent tokens, so a partial sub-chunk leaves the state alone).
__device__ void lap_stage(const LapBwdArgs &a, LapStage &st, int b, int h, int t0, int n, bool bwd, int64_t row_base) {
  constexpr int kPer = 8, kRounds = kLC * 64 / (kLT * kPer);
  const int tid = threadIdx.x;
  float xb = 0.f;
  if (tid < kLC && tid < n) xb = load_any(a.beta, a.beta_dt, b * a.s_b.b + h * a.s_b.h + (int64_t)(t0 + tid) * a.s_b.t);
#pragma unroll 1
  for (int rd = 0; rd < kRounds; ++rd) {
  float xk[kPer], xmk[kPer], xq[kPer], xmq[kPer], xv[kPer], xl[kPer], xo[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int idx = tid + (rd * kPer + i) * kLT, r = idx >> 6, c = idx & 63, t = t0 + r;
    const bool ok = r < n;
    xk[i] = xmk[i] = xq[i] = xmq[i] = xv[i] = xo[i] = 0.f;
    xl[i] = 0.f;
    if (ok && c < a.D) {
      xk[i] = load_any(a.tk, a.in_dt, b * a.s_tk.b + h * a.s_tk.h + (int64_t)t * a.s_tk.t + c);
      if (a.mk) xmk[i] = load_any(a.mk, a.in_dt, b * a.s_mk.b + h * a.s_mk.h + (int64_t)t * a.s_mk.t + c);
      if (bwd) {
        xq[i] = load_any(a.tq, a.in_dt, b * a.s_tq.b + h * a.s_tq.h + (int64_t)t * a.s_tq.t + c);
        if (a.mq) xmq[i] = load_any(a.mq, a.in_dt, b * a.s_mq.b + h * a.s_mq.h + (int64_t)t * a.s_mq.t + c);
      }
    }
    if (ok && c < a.Dv) {
      xv[i] = load_any(a.v, a.in_dt, b * a.s_v.b + h * a.s_v.h + (int64_t)t * a.s_v.t + c);
      xl[i] = load_any(a.ld, a.in_dt, b * a.s_ld.b + h * a.s_ld.h + (int64_t)t * a.s_ld.t + c);
      if (bwd) xo[i] = a.dout[row_base + (int64_t)t * a.Dv + c];
    }
  }
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int idx = tid + (rd * kPer + i) * kLT, r = idx >> 6, c = idx & 63;
    const bool ok = r < n;
    float s, co, mag = __expf(xmk[i]);
    sincosf(xk[i], &s, &co);
    st.kc[r][c] = (ok && c < a.D) ? mag * co : 0.f;
    st.ks[r][c] = (ok && c < a.D) ? mag * s : 0.f;
    if (bwd) {
      mag = __expf(xmq[i]);
      sincosf(xq[i], &s, &co);
      st.qc[r][c] = (ok && c < a.D) ? mag * co : 0.f;
      st.qs[r][c] = (ok && c < a.D) ? mag * s : 0.f;
      st.dout[r][c] = xo[i];
    }
    st.v[r][c] = xv[i];
    const bool live = ok && c < a.Dv;
    const float r_ = live ? __expf(fmaxf(xl[i], kLogFloor)) : 1.f;
    st.r[r][c] = r_;
    st.rg[r][c] = (live && xl[i] > kLogFloor) ? r_ : 0.f;
  }
  }
  if (tid < kLC) st.beta[tid] = xb;
}

// One forward token (rows row0 .. row0 + 15 of this warp; lane l stands for row
// row0 + l % 16): e, u = beta e, S = diag(r) S + u kap^T.  Returns u for this lane's row
// and e through *e_out.
__device__ __forceinline__ float lap_fwd_token(float (&S)[kRW], float (*red)[4][64], const LapStage &st, int r,
                                               int j, int cb, int row0, int lane, float invD, float *e_out) {
  const float kap = (j & 1) ? st.ks[r][j >> 1] : st.kc[r][j >> 1];
  float x[kRW];
#pragma unroll
  for (int i = 0; i < kRW; ++i) x[i] = S[i] * kap;
  const float rsum = rs_rows<kRW>(x, lane);
  const int o = row0 + (lane & (kRW - 1));
  if (lane < kRW) red[0][cb][o] = rsum;
  __syncthreads();
  const float skr = red[0][0][o] + red[0][1][o] + red[0][2][o] + red[0][3][o];
  const float e = st.v[r][o] - skr * invD;
  const float u = st.beta[r] * e;
#pragma unroll
  for (int i = 0; i < kRW; ++i) S[i] = fmaf(__shfl_sync(0xffffffffu, u, i), kap, st.r[r][row0 + i] * S[i]);
  *e_out = e;
  return u;
}

__global__ void __launch_bounds__(kLT, 1) laplace_bwd_kernel(LapBwdArgs a) {
  extern __shared__ __align__(16) uint8_t lsm[];
  LapStage &st = *reinterpret_cast<LapStage *>(lsm);
  float(*red)[2][4][64] = reinterpret_cast<float(*)[2][4][64]>(lsm + sizeof(LapStage));   // [par][which][cb][row]
  float(*colb)[2][2][128] = reinterpret_cast<float(*)[2][2][128]>(
      lsm + sizeof(LapStage) + sizeof(float) * 2 * 2 * 4 * 64);  // [par][row group][q][j]
  float(*pbeta)[2] = reinterpret_cast<float(*)[2]>(
      lsm + sizeof(LapStage) + sizeof(float) * (2 * 2 * 4 * 64 + 2 * 2 * 2 * 128));  // [par][row group]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rh = blockIdx.x % a.nhalf, rg = warp >> 2, cb = warp & 3, j = 32 * cb + lane;
  const int row0 = 32 * rh + kRW * rg;
  const int bh = blockIdx.x / a.nhalf, b = bh / a.H, h = bh % a.H;
  const int L = a.L, D = a.D, Dv = a.Dv, F = 2 * D;
  const bool col_ok = j < F;
  const float invD = 1.0f / (float)D;
  const int nsc = (L + kLC - 1) / kLC;
  const int64_t row_base = (int64_t)bh * L * Dv;
  const int64_t st_base = (int64_t)bh * Dv * F;
  float *ckpt = a.ckpt + (int64_t)bh * nsc * Dv * F;
  float *scr = a.scratch + (int64_t)bh * (kLC + 1) * Dv * F;

  float S[kRW], dS[kRW];
#pragma unroll
  for (int i = 0; i < kRW; ++i) {
    const int o = row0 + i;
    S[i] = (a.state_in && col_ok && o < Dv) ? a.state_in[st_base + (int64_t)o * F + j] : 0.f;
  }

  // ---- pass 1: forward, state at every sub-chunk start to the checkpoints
  int par = 0;
  for (int sc = 0; sc < nsc; ++sc) {
    const int t0 = sc * kLC, n = min(kLC, L - t0);
#pragma unroll
    for (int i = 0; i < kRW; ++i) {
      const int o = row0 + i;
      if (col_ok && o < Dv) ckpt[((int64_t)sc * Dv + o) * F + j] = S[i];
    }
    __syncthreads();
    lap_stage(a, st, b, h, t0, n, false, row_base);
    __syncthreads();
    for (int r = 0; r < n; ++r, par ^= 1) {
      float e;
      lap_fwd_token(S, red[par], st, r, j, cb, row0, lane, invD, &e);
    }
  }

  // ---- pass 2: sub-chunks backwards
#pragma unroll
  for (int i = 0; i < kRW; ++i) {
    const int o = row0 + i;
    dS[i] = (a.dstate_out && col_ok && o < Dv) ? a.dstate_out[st_base + (int64_t)o * F + j] : 0.f;
  }
  int pend_t = -1, pend_par = 0;
  float pend_kc = 0.f, pend_ks = 0.f, pend_qc = 0.f, pend_qs = 0.f;
  auto finish = [&](int t, int pp, float kc, float ks, float qc, float qs) {
    // even lane: channel j / 2 (own = cos column, partner = sin column); this row half's
    // part of the gradients (its two row groups summed in order; outputs zeroed by the
    // entry point, so the two halves' additions commute exactly)
    const float dk = colb[pp][0][0][j] + colb[pp][1][0][j];
    const float dq = (colb[pp][0][1][j] + colb[pp][1][1][j]) * invD;
    const float dk2 = __shfl_xor_sync(0xffffffffu, dk, 1), dq2 = __shfl_xor_sync(0xffffffffu, dq, 1);
    if (rg == 0 && !(j & 1) && col_ok) {  // one row group writes the CTA's sums
      const int64_t gi = ((int64_t)bh * L + t) * D + (j >> 1);
      atomicAdd(a.dtk + gi, -ks * dk + kc * dk2);
      atomicAdd(a.dmk + gi, kc * dk + ks * dk2);
      atomicAdd(a.dtq + gi, -qs * dq + qc * dq2);
      atomicAdd(a.dmq + gi, qc * dq + qs * dq2);
    }
    if (tid == 32 * 4) atomicAdd(&a.dbeta[(int64_t)bh * L + t], pbeta[pp][0] + pbeta[pp][1]);
  };
  for (int sc = nsc - 1; sc >= 0; --sc) {
    const int t0 = sc * kLC, n = min(kLC, L - t0);
    // the sub-chunk's states: checkpoint -> scratch slot 0, S_t -> slot r + 1
#pragma unroll
    for (int i = 0; i < kRW; ++i) {
      const int o = row0 + i;
      S[i] = (col_ok && o < Dv) ? ckpt[((int64_t)sc * Dv + o) * F + j] : 0.f;
      if (col_ok && o < Dv) scr[(int64_t)o * F + j] = S[i];
    }
    __syncthreads();
    lap_stage(a, st, b, h, t0, n, true, row_base);
    __syncthreads();
    for (int r = 0; r < n; ++r, par ^= 1) {
      float e;
      const float u = lap_fwd_token(S, red[par], st, r, j, cb, row0, lane, invD, &e);
      if (cb == 0 && lane < kRW) {
        st.u[r][row0 + lane] = u;
        st.e[r][row0 + lane] = e;
      }
#pragma unroll
      for (int i = 0; i < kRW; ++i) {
        const int o = row0 + i;
        if (col_ok && o < Dv) scr[((int64_t)(r + 1) * Dv + o) * F + j] = S[i];
      }
    }
    __syncthreads();  // u, e of the sub-chunk are in the stage
    for (int r = n - 1; r >= 0; --r, par ^= 1) {
      const int t = t0 + r;
      float Sp[kRW];
#pragma unroll
      for (int i = 0; i < kRW; ++i) {
        const int o = row0 + i;
        Sp[i] = (col_ok && o < Dv) ? scr[((int64_t)r * Dv + o) * F + j] : 0.f;
      }
      const float kap = (j & 1) ? st.ks[r][j >> 1] : st.kc[r][j >> 1];
      const float xi = (j & 1) ? st.qs[r][j >> 1] : st.qc[r][j >> 1];
      float pq = 0.f, pw = 0.f, x1[kRW], x2[kRW];
#pragma unroll
      for (int i = 0; i < kRW; ++i) {
        const float dO = st.dout[r][row0 + i];
        dS[i] = fmaf(dO * invD, xi, dS[i]);
        pq = fmaf(S[i], dO, pq);
        pw = fmaf(dS[i], st.u[r][row0 + i], pw);
        x1[i] = dS[i] * kap;
        x2[i] = dS[i] * Sp[i];
      }
      const float s1 = rs_rows<kRW>(x1, lane), s2 = rs_rows<kRW>(x2, lane);
      const int o = row0 + (lane & (kRW - 1));
      if (lane < kRW) {
        red[par][0][cb][o] = s1;
        red[par][1][cb][o] = s2;
      }
      __syncthreads();
      if (pend_t >= 0) finish(pend_t, pend_par, pend_kc, pend_ks, pend_qc, pend_qs);
      const float du = red[par][0][0][o] + red[par][0][1][o] + red[par][0][2][o] + red[par][0][3][o];
      const float dr = red[par][1][0][o] + red[par][1][1][o] + red[par][1][2][o] + red[par][1][3][o];
      const float de = st.beta[r] * du;
      if (cb == 0) {
        if (lane < kRW && o < Dv) {
          a.dv[row_base + (int64_t)t * Dv + o] = de;
          a.dld[row_base + (int64_t)t * Dv + o] = dr * st.rg[r][o];
        }
        float p = (lane < kRW && o < Dv) ? du * st.e[r][o] : 0.f;
#pragma unroll
        for (int o2 = 16; o2 >= 1; o2 >>= 1) p += __shfl_xor_sync(0xffffffffu, p, o2);
        if (lane == 0) pbeta[par][rg] = p;  // summed over the row groups by finish
      }
      float pk = 0.f;
#pragma unroll
      for (int i = 0; i < kRW; ++i) {
        const float de_i = __shfl_sync(0xffffffffu, de, i);
        dS[i] = fmaf(-de_i * invD, kap, st.r[r][row0 + i] * dS[i]);
        pk = fmaf(Sp[i], de_i, pk);
        S[i] = Sp[i];
      }
      colb[par][rg][0][j] = pw - pk * invD;
      colb[par][rg][1][j] = pq;
      pend_t = t;
      pend_par = par;
      pend_kc = st.kc[r][j >> 1];
      pend_ks = st.ks[r][j >> 1];
      pend_qc = st.qc[r][j >> 1];
      pend_qs = st.qs[r][j >> 1];
    }
    __syncthreads();  // the stage is reloaded next
  }
  if (pend_t >= 0) finish(pend_t, pend_par, pend_kc, pend_ks, pend_qc, pend_qs);
  if (a.dstate_in) {
#pragma unroll
    for (int i = 0; i < kRW; ++i) {
      const int o = row0 + i;
      if (col_ok && o < Dv) a.dstate_in[st_base + (int64_t)o * F + j] = dS[i];
    }
  }
}


// ---- small heads (2 D <= 32 key features, Dv <= 32 rows): one warp per (b, h) unit.
// Lane j holds column j of S and dS for all ROWS rows in registers, so the column sums
// (the key / query gradients) are complete in each lane and the row sums are warp
// reduce-scatters: no block barrier, no atomics; two units per CTA, so that few units
// still spread over many SMs.  The reference
// module's default head (d_k = 16) runs here; the CTA kernel above would leave seven of
// its eight warps on padding at that size.
constexpr int kWarpUnits = 2;
constexpr unsigned kFull = 0xffffffffu;


// Raw per-token values of one lane: its key (and query) channel, its row's v and log r,
// beta.  Loaded a token ahead of their use.
struct LapTok {
  float tk, mk, tq, mq, v, ld, beta, dout;
};

__device__ __forceinline__ LapTok lap_tok_load(const LapBwdArgs &a, int b, int h, int t, int c, bool col_ok,
                                              int ro, bool row_ok, bool bwd, int64_t row_base) {
  LapTok x{0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (col_ok) {
    x.tk = load_any(a.tk, a.in_dt, b * a.s_tk.b + h * a.s_tk.h + (int64_t)t * a.s_tk.t + c);
    if (a.mk) x.mk = load_any(a.mk, a.in_dt, b * a.s_mk.b + h * a.s_mk.h + (int64_t)t * a.s_mk.t + c);
    if (bwd) {
      x.tq = load_any(a.tq, a.in_dt, b * a.s_tq.b + h * a.s_tq.h + (int64_t)t * a.s_tq.t + c);
      if (a.mq) x.mq = load_any(a.mq, a.in_dt, b * a.s_mq.b + h * a.s_mq.h + (int64_t)t * a.s_mq.t + c);
    }
  }
  if (row_ok) {
    x.v = load_any(a.v, a.in_dt, b * a.s_v.b + h * a.s_v.h + (int64_t)t * a.s_v.t + ro);
    x.ld = load_any(a.ld, a.in_dt, b * a.s_ld.b + h * a.s_ld.h + (int64_t)t * a.s_ld.t + ro);
    if (bwd) x.dout = a.dout[row_base + (int64_t)t * a.Dv + ro];
  }
  x.beta = load_any(a.beta, a.beta_dt, b * a.s_b.b + h * a.s_b.h + (int64_t)t * a.s_b.t);
  return x;
}

// |k| (cos, sin) of the lane's channel.
__device__ __forceinline__ void lap_phasor(float th, float lm, bool col_ok, float *pc, float *ps) {
  float sn, cs;
  sincosf(th, &sn, &cs);
  const float mag = __expf(lm);
  *pc = col_ok ? mag * cs : 0.f;
  *ps = col_ok ? mag * sn : 0.f;
}

// Per unit: checkpoints (NSC states), the sub-chunk's states (kLC + 1), and its u, e.
template <int ROWS>
__host__ __device__ constexpr size_t lap_warp_unit_floats(size_t nsc) {
  return (nsc + kLC + 1) * (size_t)ROWS * 32 + 2 * kLC * 32;
}

template <int ROWS>
__global__ void __launch_bounds__(32 * kWarpUnits) laplace_bwd_warp_kernel(LapBwdArgs a, int units) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x * kWarpUnits + warp;
  if (bh >= units) return;  // the whole warp: nothing below synchronises the block
  const int b = bh / a.H, h = bh % a.H;
  const int L = a.L, D = a.D, Dv = a.Dv, F = 2 * D;
  const int j = lane, c = j >> 1, ro = lane & (ROWS - 1);
  const bool col_ok = j < F, row_ok = ro < Dv, row_lane = lane < ROWS && row_ok;
  const float invD = 1.0f / (float)D;
  const int nsc = (L + kLC - 1) / kLC;
  const int64_t row_base = (int64_t)bh * L * Dv;
  const int64_t st_base = (int64_t)bh * Dv * F;
  constexpr int SS = ROWS * 32;
  float *ckpt = a.ckpt + (int64_t)bh * lap_warp_unit_floats<ROWS>(nsc);
  float *scr = ckpt + (int64_t)nsc * SS;
  float *ue = scr + (int64_t)(kLC + 1) * SS;  // u: [r][32], e: [kLC + r][32]

  float S[ROWS], dS[ROWS];
#pragma unroll
  for (int i = 0; i < ROWS; ++i) S[i] = (a.state_in && col_ok && i < Dv) ? a.state_in[st_base + (int64_t)i * F + j] : 0.f;

  // one forward token: returns u and e of row ro
  auto fwd = [&](const LapTok &x, float kap, float *e_out) {
    float xx[ROWS];
#pragma unroll
    for (int i = 0; i < ROWS; ++i) xx[i] = S[i] * kap;
    const float skr = rs_rows<ROWS>(xx, lane);
    const float e = x.v - skr * invD;
    const float u = x.beta * e;
    const float r = row_ok ? __expf(fmaxf(x.ld, kLogFloor)) : 1.f;
#pragma unroll
    for (int i = 0; i < ROWS; ++i) S[i] = fmaf(__shfl_sync(kFull, u, i), kap, __shfl_sync(kFull, r, i) * S[i]);
    *e_out = e;
    return u;
  };

  // ---- pass 1: forward, checkpoints at sub-chunk starts
  LapTok nx = L > 0 ? lap_tok_load(a, b, h, 0, c, col_ok, ro, row_ok, false, row_base) : LapTok{};
  for (int t = 0; t < L; ++t) {
    const LapTok x = nx;
    if (t + 1 < L) nx = lap_tok_load(a, b, h, t + 1, c, col_ok, ro, row_ok, false, row_base);
    if (t % kLC == 0) {
#pragma unroll
      for (int i = 0; i < ROWS; ++i) ckpt[(int64_t)(t / kLC) * SS + i * 32 + lane] = S[i];
    }
    float kc, ks, e;
    lap_phasor(x.tk, x.mk, col_ok, &kc, &ks);
    fwd(x, (j & 1) ? ks : kc, &e);
  }

  // ---- pass 2: sub-chunks backwards
#pragma unroll
  for (int i = 0; i < ROWS; ++i)
    dS[i] = (a.dstate_out && col_ok && i < Dv) ? a.dstate_out[st_base + (int64_t)i * F + j] : 0.f;
  for (int sc = nsc - 1; sc >= 0; --sc) {
    const int t0 = sc * kLC, n = min(kLC, L - t0);
#pragma unroll
    for (int i = 0; i < ROWS; ++i) {
      S[i] = ckpt[(int64_t)sc * SS + i * 32 + lane];
      scr[i * 32 + lane] = S[i];
    }
    nx = lap_tok_load(a, b, h, t0, c, col_ok, ro, row_ok, false, row_base);
    for (int r = 0; r < n; ++r) {
      const LapTok x = nx;
      if (r + 1 < n) nx = lap_tok_load(a, b, h, t0 + r + 1, c, col_ok, ro, row_ok, false, row_base);
      float kc, ks, e;
      lap_phasor(x.tk, x.mk, col_ok, &kc, &ks);
      const float u = fwd(x, (j & 1) ? ks : kc, &e);
      if (lane < ROWS) {
        ue[r * 32 + lane] = u;
        ue[(kLC + r) * 32 + lane] = e;
      }
#pragma unroll
      for (int i = 0; i < ROWS; ++i) scr[(int64_t)(r + 1) * SS + i * 32 + lane] = S[i];
    }
    nx = lap_tok_load(a, b, h, t0 + n - 1, c, col_ok, ro, row_ok, true, row_base);
    for (int r = n - 1; r >= 0; --r) {
      const int t = t0 + r;
      const LapTok x = nx;
      if (r > 0) nx = lap_tok_load(a, b, h, t - 1, c, col_ok, ro, row_ok, true, row_base);
      float Sp[ROWS];
#pragma unroll
      for (int i = 0; i < ROWS; ++i) Sp[i] = scr[(int64_t)r * SS + i * 32 + lane];
      float kc, ks, qc, qs;
      lap_phasor(x.tk, x.mk, col_ok, &kc, &ks);
      lap_phasor(x.tq, x.mq, col_ok, &qc, &qs);
      const float kap = (j & 1) ? ks : kc, xi = (j & 1) ? qs : qc;
      const float u_r = ue[r * 32 + ro], e_r = ue[(kLC + r) * 32 + ro];
      const float rr = row_ok ? __expf(fmaxf(x.ld, kLogFloor)) : 1.f;
      const float rg = (row_ok && x.ld > kLogFloor) ? rr : 0.f;
      float pq = 0.f, pw = 0.f, x1[ROWS], x2[ROWS];
#pragma unroll
      for (int i = 0; i < ROWS; ++i) {
        const float dO = __shfl_sync(kFull, x.dout, i);
        dS[i] = fmaf(dO * invD, xi, dS[i]);
        pq = fmaf(S[i], dO, pq);
        pw = fmaf(dS[i], __shfl_sync(kFull, u_r, i), pw);
        x1[i] = dS[i] * kap;
        x2[i] = dS[i] * Sp[i];
      }
      const float du = rs_rows<ROWS>(x1, lane);
      const float dr = rs_rows<ROWS>(x2, lane);
      const float de = x.beta * du;
      if (row_lane) {
        a.dv[row_base + (int64_t)t * Dv + ro] = de;
        a.dld[row_base + (int64_t)t * Dv + ro] = dr * rg;
      }
      float p = row_lane ? du * e_r : 0.f;
#pragma unroll
      for (int o2 = 16; o2 >= 1; o2 >>= 1) p += __shfl_xor_sync(kFull, p, o2);
      if (lane == 0) a.dbeta[(int64_t)bh * L + t] = p;
      float pk = 0.f;
#pragma unroll
      for (int i = 0; i < ROWS; ++i) {
        const float de_i = __shfl_sync(kFull, de, i);
        dS[i] = fmaf(-de_i * invD, kap, __shfl_sync(kFull, rr, i) * dS[i]);
        pk = fmaf(Sp[i], de_i, pk);
        S[i] = Sp[i];
      }
      // column sums are complete: this lane's channel (pair with the neighbouring lane)
      const float dk = pw - pk * invD, dq = pq * invD;
      const float dk2 = __shfl_xor_sync(kFull, dk, 1), dq2 = __shfl_xor_sync(kFull, dq, 1);
      if (!(j & 1) && col_ok) {
        const int64_t gi = ((int64_t)bh * L + t) * D + c;
        a.dtk[gi] = -ks * dk + kc * dk2;
        a.dmk[gi] = kc * dk + ks * dk2;
        a.dtq[gi] = -qs * dq + qc * dq2;
        a.dmq[gi] = qc * dq + qs * dq2;
      }
    }
  }
  if (a.dstate_in) {
#pragma unroll
    for (int i = 0; i < ROWS; ++i)
      if (col_ok && i < Dv) a.dstate_in[st_base + (int64_t)i * F + j] = dS[i];
  }
}

}  // namespace
}  // namespace dp

extern "C" size_t dp_laplace_bwd_workspace_size(int B, int H, int L, int D, int Dv) {
  if (B <= 0 || H <= 0 || L <= 0 || D <= 0 || Dv <= 0) return 0;
  const size_t nsc = ((size_t)L + dp::kLC - 1) / dp::kLC;
  if (2 * D <= 32 && Dv <= 32)  // one warp per unit
    return (size_t)B * H * (Dv <= 16 ? dp::lap_warp_unit_floats<16>(nsc) : dp::lap_warp_unit_floats<32>(nsc)) *
           sizeof(float);
  return (size_t)B * H * (nsc + dp::kLC + 1) * Dv * 2 * D * sizeof(float);
}

extern "C" int dp_laplace_bwd(const void *theta_k, const void *logmag_k, const void *theta_q, const void *logmag_q,
                              const void *v, const void *log_decay, const void *beta, int in_dtype, int beta_dtype,
                              const float *state_in, const float *grad_out, const float *grad_state_out,
                              float *grad_theta_k, float *grad_logmag_k, float *grad_theta_q, float *grad_logmag_q,
                              float *grad_v, float *grad_log_decay, float *grad_beta, float *grad_state_in, int B,
                              int H, int L, int D, int Dv, const int64_t *strides, void *workspace,
                              size_t workspace_bytes, void *stream) {
  using namespace dp;
  DP_REQUIRE(B >= 0 && H >= 0 && L >= 0, DP_ERR_INVALID_ARGUMENT, "dp_laplace_bwd: negative size");
  DP_REQUIRE(D >= 1 && Dv >= 1, DP_ERR_INVALID_ARGUMENT, "dp_laplace_bwd: D and Dv must be >= 1");
  DP_REQUIRE(D <= 64 && Dv <= 64, DP_ERR_UNSUPPORTED, "dp_laplace_bwd: D and Dv must be <= 64");
  DP_REQUIRE(valid_dtype(in_dtype) && valid_dtype(beta_dtype), DP_ERR_INVALID_ARGUMENT,
             "dp_laplace_bwd: bad dtype code");
  if (B == 0 || H == 0) return DP_OK;
  DP_REQUIRE(strides, DP_ERR_INVALID_ARGUMENT, "dp_laplace_bwd: null strides");
  if (L > 0) {
    DP_REQUIRE(theta_k && theta_q && v && log_decay && beta && grad_out && grad_theta_k && grad_logmag_k &&
                   grad_theta_q && grad_logmag_q && grad_v && grad_log_decay && grad_beta,
               DP_ERR_INVALID_ARGUMENT, "dp_laplace_bwd: null pointer");
    DP_REQUIRE(workspace && workspace_bytes >= dp_laplace_bwd_workspace_size(B, H, L, D, Dv), DP_ERR_WORKSPACE,
               "dp_laplace_bwd: workspace too small (dp_laplace_bwd_workspace_size)");
    const cudaError_t e = cudaMemsetAsync(grad_beta, 0, (size_t)B * H * L * sizeof(float), as_stream(stream));
    if (e != cudaSuccess) return set_error(DP_ERR_CUDA, std::string("dp_laplace_bwd: memset: ") + cudaGetErrorString(e));
  }
  LapBwdArgs a{};
  a.tk = theta_k;
  a.mk = logmag_k;
  a.tq = theta_q;
  a.mq = logmag_q;
  a.v = v;
  a.ld = log_decay;
  a.beta = beta;
  a.in_dt = in_dtype;
  a.beta_dt = beta_dtype;
  SeqStrides *ss[7] = {&a.s_tk, &a.s_mk, &a.s_tq, &a.s_mq, &a.s_v, &a.s_ld, &a.s_b};
  for (int i = 0; i < 7; ++i) *ss[i] = SeqStrides{strides[3 * i], strides[3 * i + 1], strides[3 * i + 2]};
  a.state_in = state_in;
  a.dout = grad_out;
  a.dstate_out = grad_state_out;
  a.dtk = grad_theta_k;
  a.dmk = grad_logmag_k;
  a.dtq = grad_theta_q;
  a.dmq = grad_logmag_q;
  a.dv = grad_v;
  a.dld = grad_log_decay;
  a.dbeta = grad_beta;
  a.dstate_in = grad_state_in;
  const size_t nsc = ((size_t)L + kLC - 1) / kLC;
  a.ckpt = static_cast<float *>(workspace);
  a.scratch = a.ckpt + (size_t)B * H * nsc * Dv * 2 * D;
  a.H = H;
  a.L = L;
  a.D = D;
  a.Dv = Dv;
  if (2 * D <= 32 && Dv <= 32) {  // small heads: one warp per unit
    const int units = B * H;
    auto kern = Dv <= 16 ? laplace_bwd_warp_kernel<16> : laplace_bwd_warp_kernel<32>;
    kern<<<(units + kWarpUnits - 1) / kWarpUnits, 32 * kWarpUnits, 0, as_stream(stream)>>>(a, units);
    return check_launch("laplace_bwd_warp_kernel");
  }
  // the key / query gradients are sums over the row halves: zeroed first
  if (L > 0) {
    float *zero[4] = {grad_theta_k, grad_logmag_k, grad_theta_q, grad_logmag_q};
    for (float *p : zero) {
      const cudaError_t e = cudaMemsetAsync(p, 0, (size_t)B * H * L * D * sizeof(float), as_stream(stream));
      if (e != cudaSuccess)
        return set_error(DP_ERR_CUDA, std::string("dp_laplace_bwd: memset: ") + cudaGetErrorString(e));
    }
  }
  a.nhalf = Dv > 32 ? 2 : 1;
  const size_t smem = sizeof(LapStage) + sizeof(float) * (2 * 2 * 4 * 64 + 2 * 2 * 2 * 128 + 2 * 2);
  cudaError_t e = cudaFuncSetAttribute(laplace_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return set_error(DP_ERR_CUDA, std::string("dp_laplace_bwd smem attr: ") + cudaGetErrorString(e));
  laplace_bwd_kernel<<<B * H * a.nhalf, kLT, smem, as_stream(stream)>>>(a);
  return check_launch("laplace_bwd_kernel");
}
