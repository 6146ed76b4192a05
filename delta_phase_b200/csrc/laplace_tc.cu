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
//
// tcgen05 (bf16 operands, fp32 TMEM accumulators) computes [K;Q] K^T, [K;Q] S0^T and the
// state update S^T += K^T W.  The per-channel triangular systems are solved in four
// 16-token blocks b with reference points Lref_b = Lam[16b - 1]:
//   f[s] = e^{Lref_b - Lam[s]} beta_s e[s]          (s in block b, the block's own scale)
//   e[m] = v[m] - e^{Lam[m-1]} B0k[m] - e^{Lam[m-1]-Lref_b} (X_b[m] + sum_{s<m in b} g[s][m] f[s])
//   out[m] = e^{Lam[m]-Lref_b} (e^{Lref_b} B0q[m] + sum_{s<=m} h[s][m] F_b[s])
// where X_b and the output sums run over earlier blocks' f, rescaled block to block by
// rho_k = e^{Lref_{k+1} - Lref_k}: warp-level tf32 MMAs with the accumulator rescaled
// between 16-token K segments.  Inside a block the solve is a plain forward substitution
// (no exponentials in the loop).  The factorisation needs |Lam[m] - Lref_b| <= 64 inside
// every block of the chunk, so every factor stays inside fp32 range; a chunk that breaks
// this (a decay of more than e^-64 within 16 tokens) takes the exact path instead, which
// forms every decay ratio as exp(difference) <= 1.
//
// One CTA of 256 threads per (batch, head, half of the value channels): rows of the state
// do not interact, so the two halves run independently.  Phases stream in two chunks ahead
// with bulk async copies; v, log-decay and beta are prefetched a chunk ahead in registers.
// Every wait is bounded.
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
constexpr float kFastRange = 64.0f;  // max |Lam[m] - Lref_b| for the factorised solve

// stage: theta_k, theta_q, logmag_k, logmag_q rows of a chunk (64 rows x 128 B each)
constexpr int ST_TK = 0, ST_TQ = kC * 128, ST_MK = 2 * kC * 128, ST_MQ = 3 * kC * 128;
constexpr int STAGE_BYTES = 4 * kC * 128;
constexpr int RG_KQ = 16 * 128;
constexpr int RG_32 = 4 * 128;
constexpr int LDG = 72;   // g, h: [s][m] fp32
constexpr int LDM = 72;   // channel-major per-(token, channel) arrays: [o][m] fp32
constexpr int LDF = 40;   // F: [s][o] fp32

constexpr int OFF_STAGE = 0;                                  // [2]
constexpr int OFF_KQ = OFF_STAGE + 2 * STAGE_BYTES;          // [K; Q] bf16 128 x 128
constexpr int OFF_S0 = OFF_KQ + 16 * RG_KQ;                  // S^T bf16 128 x 32
constexpr int OFF_W = OFF_S0 + 16 * RG_32;                   // W bf16 64 x 32
constexpr int OFF_G = OFF_W + 8 * RG_32;                     // g[s][m]
constexpr int OFF_H = OFF_G + kC * LDG * 4;                  // h[s][m]
constexpr int OFF_VF = OFF_H + kC * LDG * 4;                 // v[o][m]
constexpr int OFF_LAM = OFF_VF + kNo * LDM * 4;              // Lam[o][m]
constexpr int OFF_EA = OFF_LAM + kNo * LDM * 4;              // e^{Lam[m]-Lref}[o][m]; e[o][m] (exact path)
constexpr int OFF_BK = OFF_EA + kNo * LDM * 4;               // B0k[o][m]
constexpr int OFF_BQ = OFF_BK + kNo * LDM * 4;               // B0q[o][m]
constexpr int OFF_F = OFF_BQ + kNo * LDM * 4;                // F[s][o]
constexpr int OFF_XB = OFF_F + kC * LDF * 4;                 // X of the next block [16][o]
constexpr int OFF_EREF = OFF_XB + 16 * LDF * 4;              // e^{Lref_b}[b][o]
constexpr int OFF_RHO = OFF_EREF + 4 * kNo * 4;              // rho_b[b][o]
constexpr int OFF_BETA = OFF_RHO + 4 * kNo * 4;
constexpr int OFF_BAR = OFF_BETA + kC * 4;
constexpr int SMEM_BYTES = OFF_BAR + 64;
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");

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

// Bulk copies of the phase / log-magnitude rows [c0, c0 + n) into a stage (one warp).
__device__ __forceinline__ void lap_issue_loads(const LapTcArgs &a, int b, int h, int c0, int n, uint8_t *stage,
                                                uint64_t *bar, int lane) {
  const bool has_mk = a.mk != nullptr, has_mq = a.mq != nullptr;
  const uint32_t bytes = (uint32_t)n * 128u * (2 + has_mk + has_mq);
  if (lane == 0) mbar_arrive_expect_tx(bar, bytes);
  __syncwarp();
  const __nv_bfloat16 *src[4] = {a.tk + b * a.s_tk.b + h * a.s_tk.h + (int64_t)c0 * a.s_tk.t,
                                 a.tq + b * a.s_tq.b + h * a.s_tq.h + (int64_t)c0 * a.s_tq.t,
                                 has_mk ? a.mk + b * a.s_mk.b + h * a.s_mk.h + (int64_t)c0 * a.s_mk.t : nullptr,
                                 has_mq ? a.mq + b * a.s_mq.b + h * a.s_mq.h + (int64_t)c0 * a.s_mq.t : nullptr};
  const int64_t st[4] = {a.s_tk.t, a.s_tq.t, a.s_mk.t, a.s_mq.t};
  const int off[4] = {ST_TK, ST_TQ, ST_MK, ST_MQ};
#pragma unroll
  for (int x = 0; x < 4; ++x) {
    if (!src[x]) continue;
    if (st[x] == 64) {
      if (lane == 0) bulk_g2s(stage + off[x], src[x], (uint32_t)(n * 128), bar);
    } else {
      for (int t = lane; t < n; t += 32) bulk_g2s(stage + off[x] + t * 128, src[x] + t * st[x], 128u, bar);
    }
  }
}

// Register prefetch of chunk c's v and log-decay slices (thread: token tid % 64, channels
// 8 (tid / 64) .. + 7 of this CTA's half) and beta (threads 0..63).  Past the end: v = 0,
// log r = 0, beta = 0 -- the reference's padding.
__device__ __forceinline__ void prefetch_vlr(const LapTcArgs &a, int b, int h, int oh, int c, int tid, uint4 &pv,
                                             uint4 &pl, float &pb) {
  const int tt = tid & 63, q4 = tid >> 6, t = c * kC + tt;
  pv = make_uint4(0, 0, 0, 0);
  pl = pv;
  pb = 0.f;
  if (t < a.L) {
    pv = __ldg(reinterpret_cast<const uint4 *>(a.v + b * a.s_v.b + h * a.s_v.h + (int64_t)t * a.s_v.t + kNo * oh + 8 * q4));
    pl = __ldg(reinterpret_cast<const uint4 *>(a.lr + b * a.s_lr.b + h * a.s_lr.h + (int64_t)t * a.s_lr.t + kNo * oh +
                                               8 * q4));
  }
  const int tb = c * kC + tid;
  if (tid < kC && tb < a.L) pb = load_beta(a.beta, a.beta_dt, b * a.s_b.b + h * a.s_b.h + (int64_t)tb * a.s_b.t);
}

__global__ void __launch_bounds__(kThreads, 1) laplace_tc_kernel(LapTcArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t *kq = smem + OFF_KQ;
  uint8_t *s0 = smem + OFF_S0;
  uint8_t *wt = smem + OFF_W;
  float *gm = reinterpret_cast<float *>(smem + OFF_G);
  float *hm = reinterpret_cast<float *>(smem + OFF_H);
  float *vfT = reinterpret_cast<float *>(smem + OFF_VF);
  float *lamT = reinterpret_cast<float *>(smem + OFF_LAM);
  float *eaT = reinterpret_cast<float *>(smem + OFF_EA);
  float *bkT = reinterpret_cast<float *>(smem + OFF_BK);
  float *bqT = reinterpret_cast<float *>(smem + OFF_BQ);
  float *fv = reinterpret_cast<float *>(smem + OFF_F);
  float *xb = reinterpret_cast<float *>(smem + OFF_XB);
  float *eref = reinterpret_cast<float *>(smem + OFF_EREF);
  float *rho = reinterpret_cast<float *>(smem + OFF_RHO);
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
      lap_issue_loads(a, b, h, c * kC, min(kC, L - c * kC), smem + OFF_STAGE + c * STAGE_BYTES, &load_bar[c], lane);
  }
  uint4 pv, pl;
  float pb;
  prefetch_vlr(a, b, h, oh, 0, tid, pv, pl, pb);
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
  const int g8 = lane >> 2, t4 = lane & 3;  // mma.sync fragment coordinates

  for (int c = 0; c < nchunks; ++c) {
    const int t0 = c * kC, nvalid = min(kC, L - t0), st = c & 1;
    uint8_t *stage = smem + OFF_STAGE + st * STAGE_BYTES;
    float *obase = a.out + b * a.s_out.b + h * a.s_out.h + (int64_t)t0 * a.s_out.t + kNo * oh;
    if (tid == 0) ok = mbar_wait(&load_bar[st], (uint32_t)((c >> 1) & 1), kTimeoutNs);
    if (__syncthreads_or(!ok)) { ok = false; break; }
    consumed = c + 1;

    // ---- L1: phasors (with magnitudes) -> [K; Q] bf16; v, log-decay, beta -> shared
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
      {
        const int tt = tid & 63, q4 = tid >> 6;
        const uint32_t vw[4] = {pv.x, pv.y, pv.z, pv.w}, lw[4] = {pl.x, pl.y, pl.z, pl.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 vv = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&vw[i]));
          const float2 ll = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&lw[i]));
          vfT[(8 * q4 + 2 * i) * LDM + tt] = vv.x;
          vfT[(8 * q4 + 2 * i + 1) * LDM + tt] = vv.y;
          lamT[(8 * q4 + 2 * i) * LDM + tt] = fmaxf(ll.x, kLogFloor);
          lamT[(8 * q4 + 2 * i + 1) * LDM + tt] = fmaxf(ll.y, kLogFloor);
        }
        if (tid < kC) bs[tid] = pb;
      }
      if (c + 1 < nchunks) prefetch_vlr(a, b, h, oh, c + 1, tid, pv, pl, pb);
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
    if (c + 2 < nchunks) {
      if (warp == 7) lap_issue_loads(a, b, h, t0 + 2 * kC, min(kC, L - t0 - 2 * kC), stage, &load_bar[st], lane);
      issued = c + 3;
    }
    // ---- decay: cumulative log-decay, block-relative factors (overlaps the MMAs)
    bool bad;
    {
      const int o = tid >> 3, p = tid & 7;  // channel o, tokens 8p .. 8p + 7
      float *lo = lamT + o * LDM + 8 * p;
      const float4 x0 = *reinterpret_cast<const float4 *>(lo), x1 = *reinterpret_cast<const float4 *>(lo + 4);
      float l[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
      for (int i = 1; i < 8; ++i) l[i] += l[i - 1];
      float tot = l[7];
#pragma unroll
      for (int d = 1; d < 8; d <<= 1) {
        const float n = __shfl_up_sync(0xffffffffu, tot, d, 8);
        if (p >= d) tot += n;
      }
      const float excl = tot - l[7];
      const float excl_prev = __shfl_up_sync(0xffffffffu, excl, 1, 8);
      const float lref = (p & 1) ? excl_prev : excl;  // Lam[16 (p / 2) - 1]
      float e[8], dev = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        l[i] += excl;
        const float d = l[i] - lref;
        e[i] = __expf(d);
        dev = fmaxf(dev, fabsf(d));
      }
      *reinterpret_cast<float4 *>(lo) = make_float4(l[0], l[1], l[2], l[3]);
      *reinterpret_cast<float4 *>(lo + 4) = make_float4(l[4], l[5], l[6], l[7]);
      float *eo = eaT + o * LDM + 8 * p;
      *reinterpret_cast<float4 *>(eo) = make_float4(e[0], e[1], e[2], e[3]);
      *reinterpret_cast<float4 *>(eo + 4) = make_float4(e[4], e[5], e[6], e[7]);
      if (p & 1) rho[(p >> 1) * kNo + o] = e[7];
      else eref[(p >> 1) * kNo + o] = __expf(lref);
      bad = !(dev <= kFastRange);
    }
    if (tid == 0) ok = mbar_wait(mma_bar, mma_phase, kTimeoutNs);
    if (__syncthreads_or(!ok)) { ok = false; break; }
    mma_phase ^= 1;
    mma_pending = false;
    const bool fast = !__syncthreads_or(bad);
    tc_fence_after();

    // ---- L4: g[s][m] = K K^T / D (rows 0..63, symmetric), h[s][m] = kap_s . xi_m / D
    //      (rows 64..127 hold (Q K^T)[m][s]); B0k, B0q channel-major from [K;Q] S0^T.
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
          if (row < 64) gm[col * LDG + row] = d[i] * inv_d;
          else hm[col * LDG + (row - 64)] = d[i] * inv_d;
        }
      }
      float d[16];
      tmem_ld16(tmem + lane_base + COL_D3 + 16 * hf, d);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int o = 16 * hf + i;
        if (row < 64) bkT[o * LDM + row] = d[i] * inv_d;
        else bqT[o * LDM + (row - 64)] = d[i] * inv_d;
      }
    }
    tc_fence_before();
    __syncthreads();

    const int so = tid >> 3, sj = tid & 7;  // solve layout: channel so, tokens m0 + sj, m0 + 8 + sj
    if (fast) {
      // ---- L5: factorised blocked solve; W written straight to its bf16 operand
      const float l63 = lamT[so * LDM + 63];
      for (int blk = 0; blk < 4; ++blk) {
        const int m0 = 16 * blk;
        {
          const float er = eref[blk * kNo + so];
          float R[2], A[2], Bt[2], y[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int m = m0 + 8 * u + sj;
            const float ap = eaT[so * LDM + m];
            const float am = (8 * u + sj == 0) ? 1.f : eaT[so * LDM + m - 1];
            R[u] = fmaf(-er * am, bkT[so * LDM + m], vfT[so * LDM + m]);
            A[u] = am;
            Bt[u] = __fdividef(bs[m], ap);
            y[u] = blk ? xb[(8 * u + sj) * LDF + so] : 0.f;
          }
#pragma unroll
          for (int s8 = 0; s8 < 16; ++s8) {
            const int uo = s8 >> 3;
            const float f_own = Bt[uo] * fmaf(-A[uo], y[uo], R[uo]);
            const float f = __shfl_sync(0xffffffffu, f_own, (lane & ~7) | (s8 & 7));
#pragma unroll
            for (int u = 0; u < 2; ++u)
              if (8 * u + sj > s8) y[u] = fmaf(gm[(m0 + s8) * LDG + m0 + 8 * u + sj], f, y[u]);
          }
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int m = m0 + 8 * u + sj;
            const float e = fmaf(-A[u], y[u], R[u]);
            fv[m * LDF + so] = Bt[u] * e;
            const float w = __expf(l63 - lamT[so * LDM + m]) * bs[m] * e;
            *reinterpret_cast<__nv_bfloat16 *>(wt + cm_off(m, so, RG_32)) = __float2bfloat16_rn(w);
          }
        }
        __syncthreads();
        if (blk < 3) {
          // X of the next block: rows 16 (blk + 1) .., warps 0..3 one 8-channel tile each
          if (warp < 4) {
            const int n0 = 8 * warp, r0 = m0 + 16;
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            for (int seg = 0; seg <= blk; ++seg) {
              if (seg > 0) {
                const float ra = rho[(seg - 1) * kNo + n0 + 2 * t4], rb = rho[(seg - 1) * kNo + n0 + 2 * t4 + 1];
                acc[0] *= ra; acc[1] *= rb; acc[2] *= ra; acc[3] *= rb;
              }
#pragma unroll
              for (int k8 = 0; k8 < 2; ++k8) {
                const int k0 = 16 * seg + 8 * k8;
                const uint32_t af[4] = {to_tf32(gm[(k0 + t4) * LDG + r0 + g8]), to_tf32(gm[(k0 + t4) * LDG + r0 + g8 + 8]),
                                        to_tf32(gm[(k0 + t4 + 4) * LDG + r0 + g8]),
                                        to_tf32(gm[(k0 + t4 + 4) * LDG + r0 + g8 + 8])};
                const uint32_t bf[2] = {to_tf32(fv[(k0 + t4) * LDF + n0 + g8]), to_tf32(fv[(k0 + t4 + 4) * LDF + n0 + g8])};
                mma_tf32_m16n8k8(acc, af, bf);
              }
            }
            const float ra = rho[blk * kNo + n0 + 2 * t4], rb = rho[blk * kNo + n0 + 2 * t4 + 1];
            xb[g8 * LDF + n0 + 2 * t4] = acc[0] * ra;
            xb[g8 * LDF + n0 + 2 * t4 + 1] = acc[1] * rb;
            xb[(g8 + 8) * LDF + n0 + 2 * t4] = acc[2] * ra;
            xb[(g8 + 8) * LDF + n0 + 2 * t4 + 1] = acc[3] * rb;
          }
          __syncthreads();
        }
      }
      // ---- L5o: outputs, 16 tiles (4 blocks x 4 channel tiles) over 8 warps
#pragma unroll 1
      for (int rep = 0; rep < 2; ++rep) {
        const int blk = rep == 0 ? (warp >> 2) : 3 - (warp >> 2);
        const int n0 = 8 * (warp & 3), r0 = 16 * blk;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int seg = 0; seg <= blk; ++seg) {
          if (seg > 0) {
            const float ra = rho[(seg - 1) * kNo + n0 + 2 * t4], rb = rho[(seg - 1) * kNo + n0 + 2 * t4 + 1];
            acc[0] *= ra; acc[1] *= rb; acc[2] *= ra; acc[3] *= rb;
          }
#pragma unroll
          for (int k8 = 0; k8 < 2; ++k8) {
            const int k0 = 16 * seg + 8 * k8;
            const int sa = k0 + t4, sb = k0 + t4 + 4, ma = r0 + g8, mb = r0 + g8 + 8;
            const uint32_t af[4] = {to_tf32(sa <= ma ? hm[sa * LDG + ma] : 0.f), to_tf32(sa <= mb ? hm[sa * LDG + mb] : 0.f),
                                    to_tf32(sb <= ma ? hm[sb * LDG + ma] : 0.f), to_tf32(sb <= mb ? hm[sb * LDG + mb] : 0.f)};
            const uint32_t bf[2] = {to_tf32(fv[sa * LDF + n0 + g8]), to_tf32(fv[sb * LDF + n0 + g8])};
            mma_tf32_m16n8k8(acc, af, bf);
          }
        }
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int m = r0 + g8 + 8 * hh;
          if (m < nvalid) {
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
              const int o = n0 + 2 * t4 + cc;
              const float val = eaT[o * LDM + m] * fmaf(eref[blk * kNo + o], bqT[o * LDM + m], acc[2 * hh + cc]);
              obase[(int64_t)m * a.s_out.t + o] = val;
            }
          }
        }
      }
    } else {
      // ---- L5x: exact path, every decay ratio formed as exp(difference) <= 1
      float *ev = eaT;
      const float *lo = lamT + so * LDM;
      for (int blk = 0; blk < 4; ++blk) {
        const int m0 = 16 * blk;
        const float lref = blk > 0 ? lo[m0 - 1] : 0.f;
        float rhs[2], xo[2], lprev[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int m = m0 + 8 * u + sj;
          const float lmm1 = m > 0 ? lo[m - 1] : 0.f;
          lprev[u] = lmm1;
          float xs = 0.f, xq = 0.f;
          for (int s = 0; s < m0; ++s) {
            const float f = fv[s * LDF + so];
            xs = fmaf(gm[s * LDG + m], f, xs);
            xq = fmaf(hm[s * LDG + m], f, xq);
          }
          rhs[u] = vfT[so * LDM + m] - __expf(lmm1) * bkT[so * LDM + m] - __expf(lmm1 - lref) * xs;
          xo[u] = __expf(lo[m] - lref) * xq;
        }
#pragma unroll
        for (int s8 = 0; s8 < 16; ++s8) {
          const int s = m0 + s8;
          const float es = __shfl_sync(0xffffffffu, rhs[s8 >> 3], (lane & ~7) | (s8 & 7));
          const float ls = lo[s];
          const float bes = bs[s] * es;
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int m = m0 + 8 * u + sj;
            if (m > s) rhs[u] -= __expf(lprev[u] - ls) * gm[s * LDG + m] * bes;
          }
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) ev[so * LDM + m0 + 8 * u + sj] = rhs[u];
        __syncwarp();
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int m = m0 + 8 * u + sj;
          const float lm = lo[m];
          float acc = __expf(lm) * bqT[so * LDM + m] + xo[u];
          for (int s = m0; s <= m; ++s) acc = fmaf(__expf(lm - lo[s]) * bs[s] * ev[so * LDM + s], hm[s * LDG + m], acc);
          if (m < nvalid) obase[(int64_t)m * a.s_out.t + so] = acc;
        }
        const float lend = lo[m0 + 15];
        const float scale = __expf(lend - lref);
        for (int s = sj; s < m0; s += 8) fv[s * LDF + so] *= scale;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int s = m0 + 8 * u + sj;
          fv[s * LDF + so] = __expf(lend - lo[s]) * bs[s] * rhs[u];
        }
        __syncwarp();
      }
      __syncthreads();
      // W = F (= exp(Lam[63] - Lam[s]) beta_s e_s) -> bf16 (64 tokens x 32 channels)
      {
        const int s = tid >> 2, o0 = 8 * (tid & 3);
        float w[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = fv[s * LDF + o0 + i];
        *reinterpret_cast<uint4 *>(wt + cm_off(s, o0, RG_32)) =
            make_uint4(pack_bf16(w[0], w[1]), pack_bf16(w[2], w[3]), pack_bf16(w[4], w[5]), pack_bf16(w[6], w[7]));
      }
    }
    // state decay in TMEM:  S^T[j][o] *= exp(Lam[63][o])
    if (warp < 4) {
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        float sv[16];
        tmem_ld16(tmem + lane_base + COL_S + 16 * u, sv);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) sv[i] *= __expf(lamT[(16 * u + i) * LDM + 63]);
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

// True if dp_laplace_fwd's arguments fit the tensor-core kernel: bf16, d_k = d_v = 64,
// 16-byte aligned inputs with strides in whole 16-byte units.
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
