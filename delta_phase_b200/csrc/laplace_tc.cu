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
// do not interact, so the two halves run independently.  Phases and log-magnitudes
// stream a chunk ahead through TMA tensor maps (tmap.cuh); v, log-decay and beta are
// prefetched a chunk ahead in registers.
// Every wait is bounded.
#include <type_traits>

#include <cstring>

#include "dp_common.cuh"
#include "tc_ptx.cuh"
#include "tmap.cuh"

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
constexpr int BAR_SOLVE = 1;   // named barrier of the solve warps 0, 4..7 (160 threads)
constexpr int BAR_PH = 2;      // named barrier of the phasor warps 1..3 (96 threads)
constexpr int BAR_L2 = 3;      // named barrier of warps 0..3 (128 threads): state operand ready

// stage: theta_k, theta_q, logmag_k, logmag_q rows of a chunk (64 rows x 128 B each)
constexpr int ST_TK = 0, ST_TQ = kC * 128, ST_MK = 2 * kC * 128, ST_MQ = 3 * kC * 128;
constexpr int STAGE_BYTES = 4 * kC * 128;
constexpr int RG_KQ = 16 * 128;
constexpr int RG_32 = 4 * 128;
constexpr int LDG = 72;   // g, h: [s][m] fp32
constexpr int LDM = 68;   // channel-major per-(token, channel) arrays: [o][m] fp32
constexpr int LDF = 40;   // F: [s][o] fp32

constexpr int KQ_BYTES = 16 * RG_KQ;
constexpr int OFF_STAGE = 0;                                  // phases of the next chunk
constexpr int OFF_KQ = OFF_STAGE + STAGE_BYTES;              // [K; Q] bf16 128 x 128, [2] (this / next chunk)
constexpr int OFF_S0 = OFF_KQ + 2 * KQ_BYTES;                // S^T bf16 128 x 32
constexpr int OFF_W = OFF_S0 + 16 * RG_32;                   // W bf16 64 x 32
constexpr int OFF_G = OFF_W + 8 * RG_32;                     // g[s][m]
constexpr int OFF_H = OFF_G + kC * LDG * 4;                  // h[s][m]
constexpr int OFF_VF = OFF_H + kC * LDG * 4;                 // v[o][m]
constexpr int OFF_LAM = OFF_VF + kNo * LDM * 4;              // Lam[o][m]
constexpr int OFF_EA = OFF_LAM + kNo * LDM * 4;              // e^{Lam[m]-Lref}[o][m]; e[o][m] (exact path)
constexpr int OFF_BK = OFF_EA + kNo * LDM * 4;               // B0k[o][m]; R[o][m] (factorised path)
constexpr int OFF_BT = OFF_BK + kNo * LDM * 4;               // e^{Lref - Lam[m]} beta_m [o][m]
constexpr int OFF_BQ = OFF_BT + kNo * LDM * 4;               // B0q[o][m]
constexpr int OFF_F = OFF_BQ + kNo * LDM * 4;                // F[s][o]
constexpr int OFF_XB = OFF_F + kC * LDF * 4;                 // X of the next block [16][o]
constexpr int OFF_EREF = OFF_XB + 16 * LDF * 4;              // e^{Lref_b}[b][o]
constexpr int OFF_RHO = OFF_EREF + 4 * kNo * 4;              // rho_b[b][o]
constexpr int OFF_EDEC = OFF_RHO + 4 * kNo * 4;             // e^{Lam[63]}[o]
constexpr int OFF_WSC = OFF_EDEC + kNo * 4;                // e^{Lam[63] - Lref_b}[b][o]
constexpr int OFF_BETA = OFF_WSC + 4 * kNo * 4;
constexpr int OFF_BAR = OFF_BETA + kC * 4;
constexpr int SMEM_BYTES = OFF_BAR + 64;
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
static_assert(OFF_VF % 16 == 0 && OFF_LAM % 16 == 0 && OFF_EA % 16 == 0 && OFF_BK % 16 == 0 && OFF_BT % 16 == 0 &&
                  OFF_F % 16 == 0 && OFF_G % 16 == 0 && OFF_BETA % 16 == 0 && (LDM * 4) % 16 == 0 &&
                  (LDF * 4) % 16 == 0 && (LDG * 4) % 16 == 0,
              "float4 accesses need 16-byte aligned rows");

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

struct LapTcArgs {
  const __nv_bfloat16 *tk, *mk, *tq, *mq, *v, *lr;
  const void *beta;
  int beta_dt;
  const float *state_in;
  float *out, *state_out;
  int H, L;
  SeqStrides s_tk, s_mk, s_tq, s_mq, s_v, s_lr, s_b, s_out;
  int *err;
  int use_tmap;           // load the stage through the tensor maps below
  ChunkMapDims mdims[4];  // theta_k, theta_q, logmag_k, logmag_q
};

// Tensor maps of theta_k, theta_q, logmag_k, logmag_q (tmap.cuh; absent log-magnitudes
// have none): one chunk of one (b, h) per copy.
struct alignas(64) LapMaps {
  CUtensorMap m[4];
};

// Copies of the phase / log-magnitude rows [c0, c0 + n) into a stage (one warp): one
// tiled TMA copy per tensor through the maps (L >= 64; rows past L arrive as zeros and
// are not used), else bulk copies (one per tensor for contiguous rows, one per row).
__device__ __forceinline__ void lap_issue_loads(const LapTcArgs &a, const LapMaps &maps, int b, int h, int c0, int n,
                                                uint8_t *stage, uint64_t *bar, int lane) {
  const bool has_mk = a.mk != nullptr, has_mq = a.mq != nullptr;
  if (a.use_tmap) {
    if (lane == 0) {
      mbar_arrive_expect_tx(bar, (uint32_t)kC * 128u * (2 + has_mk + has_mq));
      tma_load_chunk(stage + ST_TK, &maps.m[0], a.mdims[0], c0, h, b, bar);
      tma_load_chunk(stage + ST_TQ, &maps.m[1], a.mdims[1], c0, h, b, bar);
      if (has_mk) tma_load_chunk(stage + ST_MK, &maps.m[2], a.mdims[2], c0, h, b, bar);
      if (has_mq) tma_load_chunk(stage + ST_MQ, &maps.m[3], a.mdims[3], c0, h, b, bar);
    }
    return;
  }
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
                                             uint4 &pl, uint32_t &pb) {
  const int tt = tid & 63, q4 = tid >> 6, t = c * kC + tt;
  pv = make_uint4(0, 0, 0, 0);
  pl = pv;
  pb = 0u;
  if (t < a.L) {
    pv = __ldg(reinterpret_cast<const uint4 *>(a.v + b * a.s_v.b + h * a.s_v.h + (int64_t)t * a.s_v.t + kNo * oh + 8 * q4));
    pl = __ldg(reinterpret_cast<const uint4 *>(a.lr + b * a.s_lr.b + h * a.s_lr.h + (int64_t)t * a.s_lr.t + kNo * oh +
                                               8 * q4));
  }
  const int tb = c * kC + tid;
  if (tid < kC && tb < a.L) pb = load_raw_scalar(a.beta, a.beta_dt, b * a.s_b.b + h * a.s_b.h + (int64_t)tb * a.s_b.t);
}

// Phasors of one chunk -> [K; Q] bf16 (rows 0..63 K, 64..127 Q, no-swizzle K-major).
// Thread: token 8 warp + lane % 8, two 16-feature segments chosen so that the 16-byte
// stores of a warp hit distinct banks.
template <bool kMag>
__device__ __forceinline__ void phasor_rows(const LapTcArgs &a, const uint8_t *stage, uint8_t *kq, int nvalid,
                                            int warp, int lane) {
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int t = 8 * warp + (lane & 7), sg = ((lane >> 3) + 2 * (lane & 7) + 4 * r) & 7;
    uint32_t kw[8], qw[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) kw[i] = qw[i] = 0u;
    if (t < nvalid) {
      const uint4 kraw = *reinterpret_cast<const uint4 *>(stage + ST_TK + t * 128 + sg * 16);
      const uint4 qraw = *reinterpret_cast<const uint4 *>(stage + ST_TQ + t * 128 + sg * 16);
      const uint32_t kr[4] = {kraw.x, kraw.y, kraw.z, kraw.w}, qr[4] = {qraw.x, qraw.y, qraw.z, qraw.w};
      uint32_t mkr[4] = {0u, 0u, 0u, 0u}, mqr[4] = {0u, 0u, 0u, 0u};
      if (kMag) {
        if (a.mk) {
          const uint4 m = *reinterpret_cast<const uint4 *>(stage + ST_MK + t * 128 + sg * 16);
          mkr[0] = m.x; mkr[1] = m.y; mkr[2] = m.z; mkr[3] = m.w;
        }
        if (a.mq) {
          const uint4 m = *reinterpret_cast<const uint4 *>(stage + ST_MQ + t * 128 + sg * 16);
          mqr[0] = m.x; mqr[1] = m.y; mqr[2] = m.z; mqr[3] = m.w;
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float s0, c0, s1, c1;
        const __nv_bfloat162 k2 = *reinterpret_cast<const __nv_bfloat162 *>(&kr[i]);
        const __nv_bfloat162 q2 = *reinterpret_cast<const __nv_bfloat162 *>(&qr[i]);
        fast_sincos(__low2float(k2), &s0, &c0);
        fast_sincos(__high2float(k2), &s1, &c1);
        if (kMag) {
          // bf16 zeros in an absent magnitude tensor give e^0 = 1
          const float2 mk = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&mkr[i]));
          const float a0 = __expf(mk.x), a1 = __expf(mk.y);
          c0 *= a0; s0 *= a0; c1 *= a1; s1 *= a1;
        }
        kw[2 * i] = pack_bf16(c0, s0);
        kw[2 * i + 1] = pack_bf16(c1, s1);
        fast_sincos(__low2float(q2), &s0, &c0);
        fast_sincos(__high2float(q2), &s1, &c1);
        if (kMag) {
          const float2 mq = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&mqr[i]));
          const float b0 = __expf(mq.x), b1 = __expf(mq.y);
          c0 *= b0; s0 *= b0; c1 *= b1; s1 *= b1;
        }
        qw[2 * i] = pack_bf16(c0, s0);
        qw[2 * i + 1] = pack_bf16(c1, s1);
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
}

// acc (+)= sum over the 16-token K segments [SEG_LO, SEG_HI) of A_seg F_seg for one 16 x 8
// tile (rows R0 .. R0 + 15, channels n0 .. n0 + 7), the accumulator rescaled by rho between
// segments.  A(m, s) = amat[s * LDG + m], masked to s <= m on the diagonal segment.  Two
// accumulators (k = 0..7 / 8..15 of each segment) halve the MMA dependency chain.
template <int SEG_LO, int SEG_HI, int R0>
__device__ __forceinline__ void seg_mma(float (&acc)[4], const float *amat, const float *fv, const float *rho, int n0,
                                        int g8, int t4) {
  float a1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int seg = SEG_LO; seg < SEG_HI; ++seg) {
    if (seg > SEG_LO) {
      const float ra = rho[(seg - 1) * kNo + n0 + 2 * t4], rb = rho[(seg - 1) * kNo + n0 + 2 * t4 + 1];
      acc[0] *= ra; acc[1] *= rb; acc[2] *= ra; acc[3] *= rb;
      a1[0] *= ra; a1[1] *= rb; a1[2] *= ra; a1[3] *= rb;
    }
    const bool diag = 16 * seg == R0;
#pragma unroll
    for (int k8 = 0; k8 < 2; ++k8) {
      const int sa = 16 * seg + 8 * k8 + t4, sb = sa + 4, ma = R0 + g8, mb = ma + 8;
      float x0 = amat[sa * LDG + ma], x1 = amat[sa * LDG + mb], x2 = amat[sb * LDG + ma], x3 = amat[sb * LDG + mb];
      if (diag) {
        x0 = sa <= ma ? x0 : 0.f;
        x1 = sa <= mb ? x1 : 0.f;
        x2 = sb <= ma ? x2 : 0.f;
        x3 = sb <= mb ? x3 : 0.f;
      }
      const uint32_t af[4] = {to_tf32(x0), to_tf32(x1), to_tf32(x2), to_tf32(x3)};
      const uint32_t bf[2] = {to_tf32(fv[sa * LDF + n0 + g8]), to_tf32(fv[sb * LDF + n0 + g8])};
      if (k8 == 0) mma_tf32_m16n8k8(acc, af, bf);
      else mma_tf32_m16n8k8(a1, af, bf);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i] += a1[i];
}

// Forward substitution of block BLK for channel o (one lane per channel):
//   f[s] = Bt[s] (R[s] - A[s] y[s]),  y[m] += g[s][m] f[s] for m > s,  y starts at X_b,
// with A[s] = e^{Lam[s-1] - Lref_b} (1 at the block's first token), Bt = e^{Lref_b - Lam[s]} beta_s.
// Writes F[s][o] = f[s].
// One instance for all four blocks (m0 at run time): the solver runs on one warp, and a
// single copy of its unrolled 16-step body stays in the instruction cache.
__device__ __noinline__ void solve_block(int o, int BLK, const float *gm, const float *rT, const float *eaT,
                                         const float *btT, const float *xb, float *fv) {
  const int m0 = 16 * BLK;
  float R[16], E[16], Bt[16], y[16], f[16];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const float4 r4 = *reinterpret_cast<const float4 *>(rT + o * LDM + m0 + 4 * c);
    const float4 e4 = *reinterpret_cast<const float4 *>(eaT + o * LDM + m0 + 4 * c);
    const float4 b4 = *reinterpret_cast<const float4 *>(btT + o * LDM + m0 + 4 * c);
    R[4 * c] = r4.x; R[4 * c + 1] = r4.y; R[4 * c + 2] = r4.z; R[4 * c + 3] = r4.w;
    E[4 * c] = e4.x; E[4 * c + 1] = e4.y; E[4 * c + 2] = e4.z; E[4 * c + 3] = e4.w;
    Bt[4 * c] = b4.x; Bt[4 * c + 1] = b4.y; Bt[4 * c + 2] = b4.z; Bt[4 * c + 3] = b4.w;
  }
#pragma unroll
  for (int k = 0; k < 16; ++k) y[k] = BLK ? xb[k * LDF + o] : 0.f;
#pragma unroll
  for (int s = 0; s < 16; ++s) {
    const float A = s ? E[s - 1] : 1.f;
    f[s] = Bt[s] * fmaf(-A, y[s], R[s]);
    if (s < 15) {
      const float *grow = gm + (m0 + s) * LDG + m0;
#pragma unroll
      for (int c4 = (s + 1) >> 2; c4 < 4; ++c4) {
        const float4 g4 = *reinterpret_cast<const float4 *>(grow + 4 * c4);
        const float gv[4] = {g4.x, g4.y, g4.z, g4.w};
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (4 * c4 + k > s) y[4 * c4 + k] = fmaf(gv[k], f[s], y[4 * c4 + k]);
      }
    }
  }
  // stores after the loop: no shared-memory store sits between the g loads of the chain
#pragma unroll
  for (int s = 0; s < 16; ++s) fv[(m0 + s) * LDF + o] = f[s];
}

__global__ void __launch_bounds__(kThreads, 1) laplace_tc_kernel(const __grid_constant__ LapTcArgs a,
                                                                  const __grid_constant__ LapMaps maps) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t *stage = smem + OFF_STAGE;
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
  float *edec = reinterpret_cast<float *>(smem + OFF_EDEC);
  float *wsc = reinterpret_cast<float *>(smem + OFF_WSC);
  float *btT = reinterpret_cast<float *>(smem + OFF_BT);
  float *bs = reinterpret_cast<float *>(smem + OFF_BETA);
  uint64_t *mma_bar = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
  uint64_t *load_bar = mma_bar + 1;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_bar + 2);
  int *last_issued = reinterpret_cast<int *>(mma_bar + 3);  // chunk of the newest stage load

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int unit = blockIdx.x >> 1, oh = blockIdx.x & 1;
  const int b = unit / a.H, h = unit % a.H;
  const int L = a.L, nchunks = (L + kC - 1) / kC;
  const float inv_d = 1.0f / 64.0f;

  if (tid == 0) {
    mbar_init(mma_bar, 1);
    mbar_init(load_bar, 1);
    *last_issued = -1;
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

  const bool has_mag = a.mk || a.mq;
  // Phasors of chunk cn -> its [K; Q] buffer by warps wfirst .. wfirst + nw - 1 (barrier
  // bar_id over them; 0 = the whole CTA), then the stage load of chunk cn + 1.
  auto next_phasors = [&](int cn, int wfirst, int nw, int bar_id) -> bool {
    bool okl = true;
    if (tid == 32 * wfirst) okl = mbar_wait(load_bar, (uint32_t)(cn & 1), kTimeoutNs);
    if (bar_id == 0 ? __syncthreads_or(!okl) : group_any(!okl, bar_id, 32 * nw)) return false;
    uint8_t *dst = smem + OFF_KQ + (cn & 1) * KQ_BYTES;
    const int nv = min(kC, L - cn * kC);
    for (int grp = warp - wfirst; grp < 8; grp += nw) {
      if (has_mag) phasor_rows<true>(a, stage, dst, nv, grp, lane);
      else phasor_rows<false>(a, stage, dst, nv, grp, lane);
    }
    fence_proxy_async_smem();
    if (bar_id == 0) __syncthreads();
    else group_sync(bar_id, 32 * nw);
    if (cn + 1 < nchunks && warp == wfirst) {
      lap_issue_loads(a, maps, b, h, (cn + 1) * kC, min(kC, L - (cn + 1) * kC), stage, load_bar, lane);
      if (lane == 0) *last_issued = cn + 1;
    }
    return true;
  };
  if (warp == 0 && nchunks > 0) {
    lap_issue_loads(a, maps, b, h, 0, min(kC, L), stage, load_bar, lane);
    if (lane == 0) *last_issued = 0;
  }
  uint4 pv, pl;
  uint32_t pb;  // raw bits of beta (converted when stored)
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
  const int g8 = lane >> 2, t4 = lane & 3;  // mma.sync fragment coordinates
  if (nchunks > 0) ok = next_phasors(0, 0, 8, 0);

  for (int c = 0; ok && c < nchunks; ++c) {
    const int t0 = c * kC, nvalid = min(kC, L - t0);
    uint8_t *kq = smem + OFF_KQ + (c & 1) * KQ_BYTES;  // phasors of this chunk (made a chunk ahead)
    float *obase = a.out + b * a.s_out.b + h * a.s_out.h + (int64_t)t0 * a.s_out.t + kNo * oh;

    // ---- L1: v, log-decay (clamped), beta from the prefetch registers -> shared
    {
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
        if (tid < kC) bs[tid] = raw_scalar_to_f32(pb, a.beta_dt);
      }
      // ---- L1p: prefetch of the next chunk's v, log-decay and beta
      if (c + 1 < nchunks) prefetch_vlr(a, b, h, oh, c + 1, tid, pv, pl, pb);
    }
    // L1 -> the decay pass reads the staged log-decay and beta of every thread
    __syncthreads();
    bool bad = false;
    if (warp < 4) {
      // ---- L2: S^T (TMEM fp32) -> bf16 operand (128 x 32), MN-major B of [K;Q] S0^T
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
      fence_proxy_async_smem();
      tc_fence_before();
      group_sync(BAR_L2, 128);
      // ---- L3: [K;Q] K^T -> D1 (M=128, N=64) and [K;Q] S0^T -> D3 (M=128, N=32), issued
      //      by one elected lane of warp 0 (the issuing thread is held for each MMA, so warp 0
      //      does no decay work)
      if (warp == 0) {
        tc_fence_after();
        const uint32_t sa = smem_u32(kq), ss = smem_u32(s0);
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t ad = make_desc(sa + kk * 256, 128, RG_KQ);
            mma_f16_ss(tmem + COL_D1, ad, make_desc(sa + kk * 256, 128, RG_KQ), idesc_bf16(128, 64, false, false),
                       kk > 0);
            mma_f16_ss(tmem + COL_D3, ad, make_desc(ss + kk * 2 * RG_32, RG_32, 128), idesc_bf16(128, 32, false, true),
                       kk > 0);
          }
          mma_commit(mma_bar);
        }
        __syncwarp();
      }
    } else {
      // ---- decay (warps 4..7, overlapping L2 and the MMAs): cumulative log-decay and the
      //      block-relative factors, 16 channels per pass
      for (int pass = 0; pass < 2; ++pass) {
          const int o = 16 * pass + 4 * (warp - 4) + (lane >> 3), p = lane & 7;  // tokens 8p .. 8p + 7
        float *lo = lamT + o * LDM + 8 * p;
        const float4 x0 = *reinterpret_cast<const float4 *>(lo), x1 = *reinterpret_cast<const float4 *>(lo + 4);
        const float4 b0 = *reinterpret_cast<const float4 *>(bs + 8 * p), b1 = *reinterpret_cast<const float4 *>(bs + 8 * p + 4);
        const float bsv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
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
        if (p == 7) edec[o] = __expf(l[7]);
        const float l63 = __shfl_sync(0xffffffffu, l[7], (lane & ~7) | 7);
        if (!(p & 1)) wsc[(p >> 1) * kNo + o] = __expf(l63 - lref);
        float bt[8];
  #pragma unroll
        for (int i = 0; i < 8; ++i) bt[i] = __fdividef(bsv[i], e[i]);
        float *bo = btT + o * LDM + 8 * p;
        *reinterpret_cast<float4 *>(bo) = make_float4(bt[0], bt[1], bt[2], bt[3]);
        *reinterpret_cast<float4 *>(bo + 4) = make_float4(bt[4], bt[5], bt[6], bt[7]);
        bad = bad || !(dev <= kFastRange);
      }
    }
    mma_pending = true;
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
      // operands of R (factorised path, K rows) gathered before any store of this phase
      float rv[16], ra[16], re[16];
      if (fast && row < 64) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int o = 16 * hf + i;
          rv[i] = vfT[o * LDM + row];
          ra[i] = (row & 15) ? eaT[o * LDM + row - 1] : 1.f;
          re[i] = eref[(row >> 4) * kNo + o];
        }
      }
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
        if (row < 64) {
          // factorised path: R[m] = v[m] - e^{Lam[m-1]} B0k[m] (e^{Lam[m-1]} = e^{Lref} A[m])
          bkT[o * LDM + row] = fast ? fmaf(-re[i] * ra[i], d[i] * inv_d, rv[i]) : d[i] * inv_d;
        }
        else bqT[o * LDM + (row - 64)] = d[i] * inv_d;
      }
    }
    tc_fence_before();
    __syncthreads();

    if (fast && warp >= 1 && warp <= 3) {
      // ---- L5p: warps 1..3 make the next chunk's phasors while the others solve this one
      if (c + 1 < nchunks && !next_phasors(c + 1, 1, 3, BAR_PH)) ok = false;
    } else if (fast) {
      // ---- L5: factorised blocked solve.  Warp 0 (lane = channel) runs the forward
      //      substitution of each block; meanwhile warps 4..7 fold the earlier blocks into X
      //      of the next block and form the previous block's outputs; after the barrier they
      //      add the newest block to X.  Barriers over these five warps only.
      const int n0 = 8 * (warp & 3);
      float xacc[4];
      auto outputs = [&](auto bc) {
        constexpr int OB = decltype(bc)::value;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        seg_mma<0, OB + 1, 16 * OB>(acc, hm, fv, rho, n0, g8, t4);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int m = 16 * OB + g8 + 8 * hh;
          if (m < nvalid) {
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
              const int o = n0 + 2 * t4 + cc;
              obase[(int64_t)m * a.s_out.t + o] =
                  eaT[o * LDM + m] * fmaf(eref[OB * kNo + o], bqT[o * LDM + m], acc[2 * hh + cc]);
            }
          }
        }
      };
      auto block_step = [&](auto bc) {
        constexpr int BLK = decltype(bc)::value;
        if (warp == 0) {
          solve_block(lane, BLK, gm, bkT, eaT, btT, xb, fv);
        } else if (warp >= 4) {
          if constexpr (BLK > 0) outputs(std::integral_constant<int, BLK - 1>{});
          if constexpr (BLK > 0 && BLK < 3) {
#pragma unroll
            for (int i = 0; i < 4; ++i) xacc[i] = 0.f;
            seg_mma<0, BLK, 16 * (BLK + 1)>(xacc, gm, fv, rho, n0, g8, t4);
            const float ra = rho[(BLK - 1) * kNo + n0 + 2 * t4], rb = rho[(BLK - 1) * kNo + n0 + 2 * t4 + 1];
            xacc[0] *= ra; xacc[1] *= rb; xacc[2] *= ra; xacc[3] *= rb;
          }
        }
        // ---- L5b: block solved; F of the block visible to the solve warps after the barrier
        group_sync(BAR_SOLVE, 160);
        if constexpr (BLK < 3) {
          if (warp >= 4) {
            if constexpr (BLK == 0) {
#pragma unroll
              for (int i = 0; i < 4; ++i) xacc[i] = 0.f;
            }
            seg_mma<BLK, BLK + 1, 16 * (BLK + 1)>(xacc, gm, fv, rho, n0, g8, t4);
            const float ra = rho[BLK * kNo + n0 + 2 * t4], rb = rho[BLK * kNo + n0 + 2 * t4 + 1];
            xb[g8 * LDF + n0 + 2 * t4] = xacc[0] * ra;
            xb[g8 * LDF + n0 + 2 * t4 + 1] = xacc[1] * rb;
            xb[(g8 + 8) * LDF + n0 + 2 * t4] = xacc[2] * ra;
            xb[(g8 + 8) * LDF + n0 + 2 * t4 + 1] = xacc[3] * rb;
          }
          // ---- L5c: X of the next block visible after the barrier
          group_sync(BAR_SOLVE, 160);
        }
      };
      block_step(std::integral_constant<int, 0>{});
      block_step(std::integral_constant<int, 1>{});
      block_step(std::integral_constant<int, 2>{});
      block_step(std::integral_constant<int, 3>{});
      // ---- L5z: last block's outputs, then W = e^{Lam[63] - Lref_b} F -> bf16 (warps 4..7)
      if (warp >= 4) {
        outputs(std::integral_constant<int, 3>{});
        const int s = (tid - 128) >> 1, o0 = 16 * (tid & 1);
#pragma unroll
        for (int hv = 0; hv < 2; ++hv) {
          const float4 f0 = *reinterpret_cast<const float4 *>(fv + s * LDF + o0 + 8 * hv);
          const float4 f1 = *reinterpret_cast<const float4 *>(fv + s * LDF + o0 + 8 * hv + 4);
          const float *ws = wsc + (s >> 4) * kNo + o0 + 8 * hv;
          *reinterpret_cast<uint4 *>(wt + cm_off(s, o0 + 8 * hv, RG_32)) =
              make_uint4(pack_bf16(f0.x * ws[0], f0.y * ws[1]), pack_bf16(f0.z * ws[2], f0.w * ws[3]),
                         pack_bf16(f1.x * ws[4], f1.y * ws[5]), pack_bf16(f1.z * ws[6], f1.w * ws[7]));
        }
      }
    } else {
      // ---- L5x: exact path, every decay ratio formed as exp(difference) <= 1
      const int so = tid >> 3, sj = tid & 7;  // channel so, tokens m0 + sj, m0 + 8 + sj
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
      // next chunk's phasors by the whole CTA
      if (c + 1 < nchunks && !next_phasors(c + 1, 0, 8, 0)) ok = false;
    }
    // state decay in TMEM:  S^T[j][o] *= exp(Lam[63][o])  (warps 4..7 on the factorised
    // path, 0..3 on the exact one; warp w reaches TMEM lanes 32 (w % 4) ..)
    if (fast ? warp >= 4 : warp < 4) {
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        float sv[16];
        tmem_ld16(tmem + lane_base + COL_S + 16 * u, sv);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) sv[i] *= edec[16 * u + i];
        tmem_st16(tmem + lane_base + COL_S + 16 * u, sv);
      }
      tmem_st_wait();
    }
    fence_proxy_async_smem();
    tc_fence_before();
    if (__syncthreads_or(!ok)) { ok = false; break; }

    // ---- L6: S^T += K^T W  (M=128, N=32, K=64)
    if (warp == 0) {
      tc_fence_after();
      const uint32_t sk = smem_u32(kq), sw = smem_u32(wt);
      if (elect_one()) {
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f16_ss(tmem + COL_S, make_desc(sk + kk * 2 * RG_KQ, RG_KQ, 128),
                     make_desc(sw + kk * 2 * RG_32, RG_32, 128), idesc_bf16(128, 32, true, true), 1u);
        mma_commit(mma_bar);
      }
      __syncwarp();
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
      // a stage load still in flight: its phase completes (waits on a finished phase return at once)
      if (*last_issued >= 0) mbar_wait(load_bar, (uint32_t)(*last_issued & 1), kTimeoutNs);
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
  LapMaps maps;
  memset(&maps, 0, sizeof(maps));
  {
    const void *base[4] = {a.tk, a.tq, a.mk, a.mq};
    const SeqStrides *st[4] = {&a.s_tk, &a.s_tq, &a.s_mk, &a.s_mq};
    auto al16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    a.use_tmap = L >= kC;
    for (int x = 0; x < 4 && a.use_tmap; ++x) {
      if (!base[x]) continue;
      a.use_tmap = al16(base[x]) && st[x]->t % 8 == 0 && st[x]->h % 8 == 0 && st[x]->b % 8 == 0 &&
                   encode_chunk_map(&maps.m[x], &a.mdims[x], base[x], B, H, L, *st[x]);
    }
  }
  laplace_tc_kernel<<<2 * B * H, kThreads, SMEM_BYTES, stream>>>(a, maps);
  return check_launch("laplace_tc_kernel");
}

}  // namespace dp
