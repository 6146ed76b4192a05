// Tensor-core (tcgen05) LaplacePhaseCore chunkwise forward for d_k = 64, d_v = 64,
// bf16 inputs, fp32 accumulation.
//
// Reference: LaplacePhaseCore.forward (delta_phase/layers.py:481-561), token-loop oracle
// forward_sequential (layers.py:563-583), mcarbonell/delta-phase v1.3.0.
//
// Recurrence per (batch, head) and value channel o (rows of the state are independent:
// each has its own decay):  e_t[o] = v_t[o] - S[o,:] kap_t / D  (pre-decay state);
//   S[o,:] = r_t[o] S[o,:] + beta_t e_t[o] kap_t;   out_t[o] = S[o,:] xi_t / D,
// kap_t = e^{sigma_k} [cos th_k, sin th_k] (interleaved), log r clamped at -80 per step.
// Per 64-token chunk with the in-chunk cumulative log-decay Lam[t][o] (Lam[-1] = 0):
//   e[m] = v[m] - e^{Lam[m-1]} B0k[m] - sum_{s<m} e^{Lam[m-1]-Lam[s]} beta_s g[s][m] e[s]
//   out[m] = e^{Lam[m]} B0q[m] + sum_{s<=m} e^{Lam[m]-Lam[s]} beta_s e[s] h[s][m]
//   S_end = e^{Lam[63]} S0 + sum_s e^{Lam[63]-Lam[s]} beta_s e[s] kap_s
// with g = K K^T / D, h[s][m] = kap_s . xi_m / D, B0k = K S0^T / D, B0q = Q S0^T / D.
// tcgen05 (bf16 operands, fp32 TMEM accumulators) computes [K;Q] K^T, [K;Q] S0^T and the
// state update S^T += K^T W.  The per-channel triangular systems run on the CUDA cores in
// four 16-token blocks: terms from earlier blocks go through a running accumulator
//   F[s][o] = e^{Lam[16b-1][o] - Lam[s][o]} beta_s e[s][o]   (rescaled block to block),
// so every decay factor that is formed is exp(non-positive) -- nothing can overflow --
// while terms inside a block use exact exp(Lam[m-1] - Lam[s]).  After the last block F is
// the state-update weight W.  The state decay e^{Lam[63]} is applied in TMEM.
//
// One CTA of 256 threads per (batch, head, half of the value channels); inputs stream in
// two chunks ahead with bulk async copies; every wait is bounded.
#include "dp_common.cuh"
#include "tc_ptx.cuh"

namespace dp {

int *device_error_ptr();

namespace {

using namespace ptx;

constexpr int kC = 64;          // tokens per chunk
constexpr int kF = 128;         // key features
constexpr int kDv = 64;         // value channels of the head
constexpr int kNo = 32;         // value channels per CTA
constexpr int kThreads = 256;
constexpr uint64_t kTimeoutNs = 2000000000ull;
constexpr float kLogFloor = -80.0f;

// stage: theta_k, theta_q, logmag_k, logmag_q rows (128 B), v and log-decay half rows (64 B)
constexpr int ST_TK = 0, ST_TQ = kC * 128, ST_MK = 2 * kC * 128, ST_MQ = 3 * kC * 128;
constexpr int ST_V = 4 * kC * 128, ST_LR = ST_V + kC * 64;
constexpr int STAGE_BYTES = ST_LR + kC * 64;
constexpr int RG_KQ = 16 * 128;
constexpr int RG_32 = 4 * 128;
constexpr int LDG = 65;   // fp32 64 x 64 matrices
constexpr int LDO = 33;   // fp32 64 x 32 matrices

constexpr int OFF_STAGE = 0;                                  // [2]
constexpr int OFF_KQ = OFF_STAGE + 2 * STAGE_BYTES;          // [K; Q] bf16 128 x 128
constexpr int OFF_S0 = OFF_KQ + 16 * RG_KQ;                  // S^T bf16 128 x 32
constexpr int OFF_W = OFF_S0 + 16 * RG_32;                   // W bf16 64 x 32
constexpr int OFF_G = OFF_W + 8 * RG_32;                     // g[s][m] fp32
constexpr int OFF_H = OFF_G + kC * LDG * 4;                  // h[s][m] fp32
constexpr int OFF_BK = OFF_H + kC * LDG * 4;                 // B0k[m][o] fp32
constexpr int OFF_BQ = OFF_BK + kC * LDO * 4;                // B0q[m][o]
constexpr int OFF_LAM = OFF_BQ + kC * LDO * 4;               // Lam[m][o]
constexpr int OFF_E = OFF_LAM + kC * LDO * 4;                // e[m][o]
constexpr int OFF_F = OFF_E + kC * LDO * 4;                  // F[s][o]
constexpr int OFF_VF = OFF_F + kC * LDO * 4;                 // v[m][o] fp32
constexpr int OFF_BETA = OFF_VF + kC * LDO * 4;
constexpr int OFF_BAR = OFF_BETA + kC * 4;
constexpr int SMEM_BYTES = OFF_BAR + 64;

constexpr uint32_t COL_S = 0, COL_D1 = 32, COL_D3 = 96, TMEM_COLS = 128;

__device__ __forceinline__ uint32_t cm_off(int r, int k, int rg) {
  return (uint32_t)((r >> 3) * rg + (k >> 3) * 128 + (r & 7) * 16 + (k & 7) * 2);
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&h);
}

__device__ __forceinline__ void fast_sincos(float x, float *s, float *c) {
  const float k = fmaf(x, 0.15915494309189535f, 12582912.0f) - 12582912.0f;
  float r = fmaf(-k, 6.28318548202514648f, x);
  r = fmaf(-k, -1.7484556e-07f, r);
  __sincosf(r, s, c);
}

__device__ __forceinline__ float load_beta(const void *p, int dt, int64_t i) {
  if (dt == DP_F32) return static_cast<const float *>(p)[i];
  if (dt == DP_BF16) return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
  return __half2float(static_cast<const __half *>(p)[i]);
}

struct LapTcArgs {
  const __nv_bfloat16 *tk, *mk, *tq, *mq, *v, *lr;
  const void *beta;
  int beta_dt;
  const float *state_in;
  float *out, *state_out;
  int H, L;
  SeqStrides s_tk, s_mk, s_tq, s_mq, s_v, s_lr, s_b, s_out;
  int *err;
};

// Bulk copies of chunk rows [c0, c0 + n) into a stage (one warp; lane 0 registers bytes).
__device__ __forceinline__ void lap_issue_loads(const LapTcArgs &a, int b, int h, int oh, int c0, int n,
                                                uint8_t *stage, uint64_t *bar, int lane) {
  const bool has_mk = a.mk != nullptr, has_mq = a.mq != nullptr;
  const uint32_t bytes = (uint32_t)n * (128u * (2 + has_mk + has_mq) + 64u * 2);
  if (lane == 0) mbar_arrive_expect_tx(bar, bytes);
  __syncwarp();
  const __nv_bfloat16 *src128[4] = {a.tk + b * a.s_tk.b + h * a.s_tk.h + (int64_t)c0 * a.s_tk.t,
                                    a.tq + b * a.s_tq.b + h * a.s_tq.h + (int64_t)c0 * a.s_tq.t,
                                    has_mk ? a.mk + b * a.s_mk.b + h * a.s_mk.h + (int64_t)c0 * a.s_mk.t : nullptr,
                                    has_mq ? a.mq + b * a.s_mq.b + h * a.s_mq.h + (int64_t)c0 * a.s_mq.t : nullptr};
  const int64_t st128[4] = {a.s_tk.t, a.s_tq.t, a.s_mk.t, a.s_mq.t};
  const int off128[4] = {ST_TK, ST_TQ, ST_MK, ST_MQ};
#pragma unroll
  for (int x = 0; x < 4; ++x) {
    if (!src128[x]) continue;
    if (st128[x] == 64) {
      if (lane == 0) bulk_g2s(stage + off128[x], src128[x], (uint32_t)(n * 128), bar);
    } else {
      for (int t = lane; t < n; t += 32) bulk_g2s(stage + off128[x] + t * 128, src128[x] + t * st128[x], 128u, bar);
    }
  }
  const __nv_bfloat16 *src64[2] = {a.v + b * a.s_v.b + h * a.s_v.h + (int64_t)c0 * a.s_v.t + kNo * oh,
                                   a.lr + b * a.s_lr.b + h * a.s_lr.h + (int64_t)c0 * a.s_lr.t + kNo * oh};
  const int64_t st64[2] = {a.s_v.t, a.s_lr.t};
  const int off64[2] = {ST_V, ST_LR};
#pragma unroll
  for (int x = 0; x < 2; ++x)
    for (int t = lane; t < n; t += 32) bulk_g2s(stage + off64[x] + t * 64, src64[x] + t * st64[x], 64u, bar);
}

__global__ void __launch_bounds__(kThreads, 1) laplace_tc_kernel(LapTcArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t *kq = smem + OFF_KQ;
  uint8_t *s0 = smem + OFF_S0;
  uint8_t *wt = smem + OFF_W;
  float *gm = reinterpret_cast<float *>(smem + OFF_G);
  float *hm = reinterpret_cast<float *>(smem + OFF_H);
  float *bk = reinterpret_cast<float *>(smem + OFF_BK);
  float *bq = reinterpret_cast<float *>(smem + OFF_BQ);
  float *lam = reinterpret_cast<float *>(smem + OFF_LAM);
  float *ev = reinterpret_cast<float *>(smem + OFF_E);
  float *fv = reinterpret_cast<float *>(smem + OFF_F);
  float *vf = reinterpret_cast<float *>(smem + OFF_VF);
  float *bs = reinterpret_cast<float *>(smem + OFF_BETA);
  uint64_t *mma_bar = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
  uint64_t *load_bar = mma_bar + 1;  // [2]
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_bar + 3);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int unit = blockIdx.x >> 1, oh = blockIdx.x & 1;
  const int b = unit / a.H, h = unit % a.H;
  const int L = a.L, nchunks = (L + kC - 1) / kC;
  const float inv_d = 1.0f / 64.0f;

  if (tid == 0) {
    mbar_init(mma_bar, 1);
    mbar_init(&load_bar[0], 1);
    mbar_init(&load_bar[1], 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int q = warp & 3;
  const uint32_t lane_base = (uint32_t)(q * 32) << 16;

  if (warp == 0) {
    for (int c = 0; c < 2 && c < nchunks; ++c)
      lap_issue_loads(a, b, h, oh, c * kC, min(kC, L - c * kC), smem + OFF_STAGE + c * STAGE_BYTES,
                      &load_bar[c], lane);
  }
  // state^T of this CTA's 32 value channels -> TMEM (lane = feature j, column = o)
  const int64_t sbase = (int64_t)unit * kDv * kF;
  if (warp < 4) {
    const int j = 32 * q + lane;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      float vals[16];
#pragma unroll
      for (int i = 0; i < 16; ++i)
        vals[i] = a.state_in ? a.state_in[sbase + (int64_t)(kNo * oh + 16 * u + i) * kF + j] : 0.f;
      tmem_st16(tmem + lane_base + COL_S + 16 * u, vals);
    }
    tmem_st_wait();
  }
  tc_fence_before();
  __syncthreads();

  uint32_t mma_phase = 0;
  bool ok = true, mma_pending = false;
  int issued = min(nchunks, 2), consumed = 0;
  // solve layout: thread (o = tid / 8, j = tid % 8) owns tokens m = j, j + 8, ... of channel o
  const int so = tid >> 3, sj = tid & 7;

  for (int c = 0; c < nchunks; ++c) {
    const int t0 = c * kC, nvalid = min(kC, L - t0), st = c & 1;
    uint8_t *stage = smem + OFF_STAGE + st * STAGE_BYTES;
    if (tid == 0) ok = mbar_wait(&load_bar[st], (uint32_t)((c >> 1) & 1), kTimeoutNs);
    if (__syncthreads_or(!ok)) { ok = false; break; }
    consumed = c + 1;

    // ---- L1: phasors (with magnitudes) -> [K; Q] bf16; v, beta, cumulative log-decay
    {
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int t = 8 * warp + (lane & 7), sg = ((lane >> 3) + 2 * (lane & 7) + 4 * r) & 7;
        const bool valid = t < nvalid;
        uint32_t kw[8], qw[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) kw[i] = qw[i] = 0u;
        if (valid) {
          const uint4 kraw = *reinterpret_cast<const uint4 *>(stage + ST_TK + t * 128 + sg * 16);
          const uint4 qraw = *reinterpret_cast<const uint4 *>(stage + ST_TQ + t * 128 + sg * 16);
          uint4 mkraw = make_uint4(0, 0, 0, 0), mqraw = mkraw;
          if (a.mk) mkraw = *reinterpret_cast<const uint4 *>(stage + ST_MK + t * 128 + sg * 16);
          if (a.mq) mqraw = *reinterpret_cast<const uint4 *>(stage + ST_MQ + t * 128 + sg * 16);
          const uint32_t kr[4] = {kraw.x, kraw.y, kraw.z, kraw.w}, qr[4] = {qraw.x, qraw.y, qraw.z, qraw.w};
          const uint32_t mkr[4] = {mkraw.x, mkraw.y, mkraw.z, mkraw.w};
          const uint32_t mqr[4] = {mqraw.x, mqraw.y, mqraw.z, mqraw.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float s0_, c0_, s1_, c1_;
            const __nv_bfloat162 k2 = *reinterpret_cast<const __nv_bfloat162 *>(&kr[i]);
            const __nv_bfloat162 m2 = *reinterpret_cast<const __nv_bfloat162 *>(&mkr[i]);
            const float a0 = a.mk ? __expf(__low2float(m2)) : 1.f, a1 = a.mk ? __expf(__high2float(m2)) : 1.f;
            fast_sincos(__low2float(k2), &s0_, &c0_);
            fast_sincos(__high2float(k2), &s1_, &c1_);
            kw[2 * i] = pack_bf16(a0 * c0_, a0 * s0_);
            kw[2 * i + 1] = pack_bf16(a1 * c1_, a1 * s1_);
            const __nv_bfloat162 q2 = *reinterpret_cast<const __nv_bfloat162 *>(&qr[i]);
            const __nv_bfloat162 n2 = *reinterpret_cast<const __nv_bfloat162 *>(&mqr[i]);
            const float b0 = a.mq ? __expf(__low2float(n2)) : 1.f, b1 = a.mq ? __expf(__high2float(n2)) : 1.f;
            fast_sincos(__low2float(q2), &s0_, &c0_);
            fast_sincos(__high2float(q2), &s1_, &c1_);
            qw[2 * i] = pack_bf16(b0 * c0_, b0 * s0_);
            qw[2 * i + 1] = pack_bf16(b1 * c1_, b1 * s1_);
          }
        }
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          *reinterpret_cast<uint4 *>(kq + cm_off(t, 16 * sg + 8 * half, RG_KQ)) =
              make_uint4(kw[4 * half], kw[4 * half + 1], kw[4 * half + 2], kw[4 * half + 3]);
          *reinterpret_cast<uint4 *>(kq + cm_off(64 + t, 16 * sg + 8 * half, RG_KQ)) =
              make_uint4(qw[4 * half], qw[4 * half + 1], qw[4 * half + 2], qw[4 * half + 3]);
        }
      }
      // v and log-decay of this CTA's channels (fp32), beta
      for (int i = tid; i < kC * kNo; i += kThreads) {
        const int t = i >> 5, o = i & 31;
        const bool valid = t < nvalid;
        vf[t * LDO + o] = valid ? __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(stage + ST_V + t * 64)[o]) : 0.f;
        lam[t * LDO + o] = valid ? fmaxf(__bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(stage + ST_LR + t * 64)[o]), kLogFloor) : 0.f;
      }
      if (tid < kC)
        bs[tid] = tid < nvalid ? load_beta(a.beta, a.beta_dt, b * a.s_b.b + h * a.s_b.h + (int64_t)(t0 + tid) * a.s_b.t) : 0.f;
    }
    __syncthreads();
    // cumulative log-decay along the chunk (one thread per channel) and the next loads
    if (tid < kNo) {
      float acc = 0.f;
      for (int t = 0; t < kC; ++t) {
        acc += lam[t * LDO + tid];
        lam[t * LDO + tid] = acc;
      }
    }
    if (c + 2 < nchunks) {
      if (warp == 7) lap_issue_loads(a, b, h, oh, t0 + 2 * kC, min(kC, L - t0 - 2 * kC), stage, &load_bar[st], lane);
      issued = c + 3;
    }
    // ---- L2: S^T (TMEM fp32) -> bf16 operand (128 x 32), MN-major B of [K;Q] S0^T
    if (warp < 4) {
      const int j = 32 * q + lane;
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        float sv[16];
        tmem_ld16(tmem + lane_base + COL_S + 16 * u, sv);
        tmem_ld_wait();
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const float *ss = sv + 8 * half;
          *reinterpret_cast<uint4 *>(s0 + cm_off(j, 16 * u + 8 * half, RG_32)) =
              make_uint4(pack_bf16(ss[0], ss[1]), pack_bf16(ss[2], ss[3]), pack_bf16(ss[4], ss[5]), pack_bf16(ss[6], ss[7]));
        }
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();

    // ---- L3: [K;Q] K^T -> D1 (M=128, N=64) and [K;Q] S0^T -> D3 (M=128, N=32)
    if (tid == 0) {
      tc_fence_after();
      const uint32_t sa = smem_u32(kq), ss = smem_u32(s0);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint64_t ad = make_desc(sa + kk * 256, 128, RG_KQ);
        mma_f16_ss(tmem + COL_D1, ad, make_desc(sa + kk * 256, 128, RG_KQ), idesc_bf16(128, 64, false, false), kk > 0);
        mma_f16_ss(tmem + COL_D3, ad, make_desc(ss + kk * 2 * RG_32, RG_32, 128), idesc_bf16(128, 32, false, true), kk > 0);
      }
      mma_commit(mma_bar);
    }
    mma_pending = true;
    if (tid == 0) ok = mbar_wait(mma_bar, mma_phase, kTimeoutNs);
    if (__syncthreads_or(!ok)) { ok = false; break; }
    mma_phase ^= 1;
    mma_pending = false;
    tc_fence_after();

    // ---- L4: g[s][m] = K K^T / D (rows 0..63), h[s][m] = kap_s . xi_m / D (rows 64..127
    //      hold (Q K^T)[m][s]); B0k, B0q from [K;Q] S0^T.  Warps 0..3 and 4..7 split columns.
    {
      const int row = 32 * q + lane, hf = warp >> 2;
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        float d[16];
        tmem_ld16(tmem + lane_base + COL_D1 + 32 * hf + 16 * u, d);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int col = 32 * hf + 16 * u + i;
          if (row < 64) gm[row * LDG + col] = d[i] * inv_d;        // g symmetric
          else hm[col * LDG + (row - 64)] = d[i] * inv_d;           // h[s = col][m = row - 64]
        }
      }
      float d[16];
      tmem_ld16(tmem + lane_base + COL_D3 + 16 * hf, d);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int o = 16 * hf + i;
        if (row < 64) bk[row * LDO + o] = d[i] * inv_d;
        else bq[(row - 64) * LDO + o] = d[i] * inv_d;
      }
    }
    tc_fence_before();
    __syncthreads();

    // ---- L5: per-channel triangular solve and outputs, four 16-token blocks
    {
      const int o = so;
      float *orow = a.out + b * a.s_out.b + h * a.s_out.h + (int64_t)t0 * a.s_out.t + kNo * oh + o;
      for (int blk = 0; blk < 4; ++blk) {
        const int m0 = 16 * blk;
        const float lref = blk > 0 ? lam[(m0 - 1) * LDO + o] : 0.f;  // Lam[16 blk - 1]
        // owned tokens of this block: m0 + sj, m0 + 8 + sj
        float rhs[2], xo[2], lprev[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int m = m0 + 8 * u + sj;
          const float lmm1 = m > 0 ? lam[(m - 1) * LDO + o] : 0.f;
          lprev[u] = lmm1;
          // terms of earlier blocks through F (exp(<= 0) factors only)
          float xs = 0.f, xq = 0.f;
          for (int s = 0; s < m0; ++s) {
            const float f = fv[s * LDO + o];
            xs = fmaf(gm[s * LDG + m], f, xs);
            xq = fmaf(hm[s * LDG + m], f, xq);
          }
          rhs[u] = vf[m * LDO + o] - __expf(lmm1) * bk[m * LDO + o] - __expf(lmm1 - lref) * xs;
          xo[u] = __expf(lam[m * LDO + o] - lref) * xq;
        }
        // in-block forward substitution (right-looking over s; owner of s = lane % 8)
#pragma unroll
        for (int s8 = 0; s8 < 16; ++s8) {
          const int s = m0 + s8;
          const int owner_u = s8 >> 3;
          const float es_own = rhs[owner_u];
          const float es = __shfl_sync(0xffffffffu, es_own, (lane & ~7) | (s8 & 7));
          const float ls = lam[s * LDO + o];
          const float bes = bs[s] * es;
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int m = m0 + 8 * u + sj;
            if (m > s) rhs[u] -= __expf(lprev[u] - ls) * gm[s * LDG + m] * bes;
          }
        }
        // e of the owned tokens; in-block output terms need e of the whole block
#pragma unroll
        for (int u = 0; u < 2; ++u) ev[(m0 + 8 * u + sj) * LDO + o] = rhs[u];
        __syncwarp();
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int m = m0 + 8 * u + sj;
          const float lm = lam[m * LDO + o];
          float acc = __expf(lm) * bq[m * LDO + o] + xo[u];
          for (int s = m0; s <= m; ++s)
            acc = fmaf(__expf(lm - lam[s * LDO + o]) * bs[s] * ev[s * LDO + o], hm[s * LDG + m], acc);
          if (m < nvalid) orow[(int64_t)m * a.s_out.t] = acc;
        }
        // F for the next block: rescale the old terms, add this block's
        const float lend = lam[(m0 + 15) * LDO + o];
        const float scale = __expf(lend - lref);
        for (int s = sj; s < m0; s += 8) fv[s * LDO + o] *= scale;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int s = m0 + 8 * u + sj;
          fv[s * LDO + o] = __expf(lend - lam[s * LDO + o]) * bs[s] * rhs[u];
        }
        __syncwarp();
      }
    }
    __syncthreads();
    // W = F (exp(Lam[63] - Lam[s]) beta_s e_s) -> bf16 (64 tokens x 32 channels)
    {
      const int s = tid >> 2, o0 = 8 * (tid & 3);
      float w[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) w[i] = fv[s * LDO + o0 + i];
      *reinterpret_cast<uint4 *>(wt + cm_off(s, o0, RG_32)) =
          make_uint4(pack_bf16(w[0], w[1]), pack_bf16(w[2], w[3]), pack_bf16(w[4], w[5]), pack_bf16(w[6], w[7]));
    }
    // state decay in TMEM:  S^T[j][o] *= exp(Lam[63][o])
    if (warp < 4) {
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        float sv[16];
        tmem_ld16(tmem + lane_base + COL_S + 16 * u, sv);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) sv[i] *= __expf(lam[63 * LDO + 16 * u + i]);
        tmem_st16(tmem + lane_base + COL_S + 16 * u, sv);
      }
      tmem_st_wait();
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();

    // ---- L6: S^T += K^T W  (M=128, N=32, K=64)
    if (tid == 0) {
      tc_fence_after();
      const uint32_t sk = smem_u32(kq), sw = smem_u32(wt);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        mma_f16_ss(tmem + COL_S, make_desc(sk + kk * 2 * RG_KQ, RG_KQ, 128),
                   make_desc(sw + kk * 2 * RG_32, RG_32, 128), idesc_bf16(128, 32, true, true), 1u);
      mma_commit(mma_bar);
    }
    mma_pending = true;
    if (tid == 0) ok = mbar_wait(mma_bar, mma_phase, kTimeoutNs);
    if (__syncthreads_or(!ok)) { ok = false; break; }
    mma_phase ^= 1;
    mma_pending = false;
    tc_fence_after();
  }

  if (!ok) {
    if (tid == 0) {
      atomicCAS(a.err, 0, DP_ERR_TIMEOUT);
      for (int k = consumed; k < issued; ++k) mbar_wait(&load_bar[k & 1], (uint32_t)((k >> 1) & 1), kTimeoutNs);
      if (mma_pending) mbar_wait(mma_bar, mma_phase, kTimeoutNs);
    }
  } else if (warp < 4) {
    const int j = 32 * q + lane;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      float sv[16];
      tmem_ld16(tmem + lane_base + COL_S + 16 * u, sv);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 16; ++i) a.state_out[sbase + (int64_t)(kNo * oh + 16 * u + i) * kF + j] = sv[i];
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, TMEM_COLS);
}

}  // namespace

// True if dp_laplace_fwd's arguments fit the tensor-core kernel.
bool laplace_tc_supported(const void *const *ptrs, int in_dt, const float *out, int D, int Dv,
                          const SeqStrides *s) {
  if (in_dt != DP_BF16 || D != 64 || Dv != 64) return false;
  auto al16 = [](const void *p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  for (int i = 0; i < 6; ++i)
    if (!al16(ptrs[i])) return false;
  if (reinterpret_cast<uintptr_t>(out) & 3) return false;
  for (int i = 0; i < 6; ++i) {
    if (!ptrs[i]) continue;
    if ((s[i].b % 8) || (s[i].h % 8) || (s[i].t % 8)) return false;
  }
  return true;
}

// ptrs: theta_k, logmag_k, theta_q, logmag_q, v, log_decay; s: their strides, beta's, out's.
int laplace_fwd_tc(const void *const *ptrs, const void *beta, int beta_dt, const float *state_in, float *out,
                   float *state_out, int B, int H, int L, const SeqStrides *s, cudaStream_t stream) {
  LapTcArgs a;
  a.tk = static_cast<const __nv_bfloat16 *>(ptrs[0]);
  a.mk = static_cast<const __nv_bfloat16 *>(ptrs[1]);
  a.tq = static_cast<const __nv_bfloat16 *>(ptrs[2]);
  a.mq = static_cast<const __nv_bfloat16 *>(ptrs[3]);
  a.v = static_cast<const __nv_bfloat16 *>(ptrs[4]);
  a.lr = static_cast<const __nv_bfloat16 *>(ptrs[5]);
  a.beta = beta;
  a.beta_dt = beta_dt;
  a.state_in = state_in;
  a.out = out;
  a.state_out = state_out;
  a.H = H;
  a.L = L;
  a.s_tk = s[0];
  a.s_mk = s[1];
  a.s_tq = s[2];
  a.s_mq = s[3];
  a.s_v = s[4];
  a.s_lr = s[5];
  a.s_b = s[6];
  a.s_out = s[7];
  a.err = device_error_ptr();
  if (!a.err) return set_error(DP_ERR_CUDA, "laplace_fwd_tc: device error word unavailable");
  cudaError_t e = cudaFuncSetAttribute(laplace_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  if (e != cudaSuccess) return set_error(DP_ERR_CUDA, std::string("laplace_tc smem attr: ") + cudaGetErrorString(e));
  laplace_tc_kernel<<<2 * B * H, kThreads, SMEM_BYTES, stream>>>(a);
  return check_launch("laplace_tc_kernel");
}

}  // namespace dp
