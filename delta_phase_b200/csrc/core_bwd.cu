// Backward of the complex delta rule (training path): gradients of the chunkwise core
// with respect to theta_k, theta_q, v, beta (or phi of the complex beta) and the initial
// state, given the gradients of the outputs and of the final state.
//
// The reference trains through PyTorch autograd of its chunkwise path
// (_chunkwise_delta_reference, delta_phase/kernels/triton_chunk_delta.py:211-252, via the
// dispatcher at :279-291; DeltaPhaseTritonFunction.backward at :271-276 raises) and of the
// complex-beta token loop (delta_phase/layers.py:346-360).  Both compute, in the real form
// of core_simt.cu, the recurrence S_t = S_{t-1} + g_t (v_t - S_{t-1} kap_t / D) w_t^T,
// o_t = S_t xi_t / D, with g = beta, w = kap (real beta) or g = 1, w = beta kap =
// (br c - bi s, br s + bi c) (complex beta, br = 1 + cos phi, bi = sin phi).
//
// Chunked adjoint (C = 32 tokens; rows = tokens; K, W, Q the key / write-key / query
// phasor rows, S^T the state at the sub-chunk start, dS^T the gradient of the state at
// its end):
//   forward again:  G = K W^T,  A = strict_lower(G) diag(g) / D,  T = (I + A)^-1,
//                   P = tril(Q W^T),  E = V - K S^T / D,  Y = T E,  U = diag(g) Y
//   dU = W dS^T + P^T dO / D;   dg += rowsum(dU o Y);   dY = diag(g) dU;   dE = T^T dY = dV
//   dA = -strict_lower(dE Y^T);  dG = dA diag(g) / D;  dg += colsum(dA o G) / D
//   dP = tril(dO U^T) / D
//   dK (read) = dG W - dE S / D;   dW = U dS + dP^T Q + dG^T K;   dQ = dO S / D + dP W
//   dS^T <- dS^T + Q^T dO / D - K^T dE / D
// then dK += dW (real beta) or R^T dW and dphi from dW (complex beta), and
// dtheta = -sin dkap_cos + cos dkap_sin.  Pass 1 runs the chunked forward and keeps the
// state at every sub-chunk start in the workspace; pass 2 walks the sub-chunks backwards.
//
// One CTA of 256 threads per (b, h); every product is a warp-level tensor-core MMA on
// fp32 shared-memory operands: the ones that carry the state and its gradient across
// sub-chunks split both operands in high and low bf16 parts (three m16n8k16 products:
// hi hi + hi lo + lo hi, 16 significant bits per operand), the sub-chunk-local gradients
// use one tf32 m16n8k8 product (see mma16).  The 32 x 32
// triangular inverse is a forward substitution by one warp (a lane per column) while the
// other warps form E.  Limits: D <= 64, Dv <= 64.
#include "dp_common.cuh"
#include "tc_ptx.cuh"

namespace dp {
namespace {

using namespace ptx;

constexpr int kBwdThreads = 256;
constexpr int kC = 32;      // tokens per sub-chunk
constexpr int kF = 128;     // key features (2 D) at most
constexpr int kDv = 64;     // value channels at most
constexpr int LD_S = 68;    // state (F x Dv), transposed
constexpr int LD_F = 132;   // C x F phasor rows
constexpr int LD_V = 68;    // C x Dv
constexpr int LD_C = 36;    // C x C
constexpr int S_FLOATS = kF * LD_S;
constexpr int F_FLOATS = kC * LD_F;
constexpr int V_FLOATS = kC * LD_V;
constexpr int C_FLOATS = kC * LD_C;
// float offsets
constexpr int O_DST = 0;
constexpr int O_ST = O_DST + S_FLOATS;
constexpr int O_K = O_ST + S_FLOATS;
constexpr int O_Q = O_K + F_FLOATS;
constexpr int O_W = O_Q + F_FLOATS;     // complex beta only
constexpr int O_V = O_W + F_FLOATS;     // V, then U
constexpr int O_DO = O_V + V_FLOATS;
constexpr int O_Y = O_DO + V_FLOATS;
constexpr int O_DU = O_Y + V_FLOATS;    // U (pass 1); dU, then dY (pass 2)
constexpr int O_DE = O_DU + V_FLOATS;   // E, then dE
constexpr int O_T = O_DE + V_FLOATS;
constexpr int O_G = O_T + C_FLOATS;
constexpr int O_P = O_G + C_FLOATS;
constexpr int O_DA = O_P + C_FLOATS;    // dG = dA diag(g) / D
constexpr int O_DP = O_DA + C_FLOATS;
constexpr int O_GV = O_DP + C_FLOATS;   // g per token (beta, or 1)
constexpr int O_BR = O_GV + kC;         // complex beta: br, bi per token
constexpr int O_BI = O_BR + kC;
constexpr int O_DG = O_BI + kC;         // d beta / d phi per token
constexpr int SMEM_FLOATS = O_DG + kC;
constexpr size_t SMEM_BYTES = SMEM_FLOATS * sizeof(float);
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");

struct BwdArgs {
  const void *tk, *tq, *v, *g;  // g: beta or phi
  int in_dt, g_dt;
  SeqStrides s_tk, s_tq, s_v, s_g;
  const float *state_in, *dout, *dstate_out;  // dout (B,H,L,Dv) contiguous; others may be null
  float *dtk, *dtq, *dv, *dg, *dstate_in;     // dtk/dtq (B,H,L,D), dv (B,H,L,Dv), dg (B,H,L)
  float *ckpt;                                // (B, H, NSC, F, Dv) states at sub-chunk starts
  int H, L, D, Dv;
};

__device__ __forceinline__ float load_any(const void *p, int dt, int64_t i) {
  if (dt == DP_F32) return static_cast<const float *>(p)[i];
  if (dt == DP_BF16) return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
  return __half2float(static_cast<const __half *>(p)[i]);
}

// d (a 16 x 16 tile as two m16n8 fragments) += X Y, X(i, k) = x[i * x_si + k * x_sk]
// (16 x K), Y(k, j) = y[k * y_sk + j * y_sj] (K x 16); tf32 products, split in high and
// low parts (hi hi + hi lo + lo hi) when SPLIT.  Unsplit products (relative error ~5e-4)
// serve the products whose result is a gradient of this sub-chunk only (dK, dQ, dA, dP,
// Y); everything that feeds the state or its gradient across sub-chunks is split (an
// error there would add up along the sequence).
// Split operand pairs in bf16: v = hi + lo with hi = bf16(v), lo = bf16(v - hi) (16
// significant bits); packs two values' parts into bf16x2 words (first value low).
__device__ __forceinline__ void split_bf16x2(float v0, float v1, uint32_t &hi, uint32_t &lo) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(v0, v1);
  const float2 hf = __bfloat1622float2(h);
  const __nv_bfloat162 l = __floats2bfloat162_rn(v0 - hf.x, v1 - hf.y);
  hi = *reinterpret_cast<const uint32_t *>(&h);
  lo = *reinterpret_cast<const uint32_t *>(&l);
}

template <int K, bool SPLIT = true>
__device__ __forceinline__ void mma16(float (&d)[2][4], const float *x, int x_si, int x_sk, const float *y, int y_sk,
                                      int y_sj, int lane) {
  const int g = lane >> 2, c = lane & 3;
  if (SPLIT) {
    // hi hi + hi lo + lo hi on bf16 m16n8k16 (half the MMAs of the tf32 m16n8k8 form per
    // k; dropped lo lo term ~2^-16 relative).  A: rows g / g + 8, k pairs (2c, 2c+1) and
    // (2c+8, 2c+9); B: the same k pairs, column g.
    static_assert(K % 16 == 0, "split products step K by 16");
    float e[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll 2
    for (int k0 = 0; k0 < K; k0 += 16) {
      const int ka = k0 + 2 * c, kb = k0 + 2 * c + 8;
      uint32_t ah[4], al[4];
      split_bf16x2(x[g * x_si + ka * x_sk], x[g * x_si + (ka + 1) * x_sk], ah[0], al[0]);
      split_bf16x2(x[(g + 8) * x_si + ka * x_sk], x[(g + 8) * x_si + (ka + 1) * x_sk], ah[1], al[1]);
      split_bf16x2(x[g * x_si + kb * x_sk], x[g * x_si + (kb + 1) * x_sk], ah[2], al[2]);
      split_bf16x2(x[(g + 8) * x_si + kb * x_sk], x[(g + 8) * x_si + (kb + 1) * x_sk], ah[3], al[3]);
#pragma unroll
      for (int n = 0; n < 2; ++n) {
        const int j = (g + 8 * n) * y_sj;
        uint32_t bh[2], bl[2];
        split_bf16x2(y[ka * y_sk + j], y[(ka + 1) * y_sk + j], bh[0], bl[0]);
        split_bf16x2(y[kb * y_sk + j], y[(kb + 1) * y_sk + j], bh[1], bl[1]);
        mma_bf16_m16n8k16(d[n], ah, bh);
        mma_bf16_m16n8k16(e[n], ah, bl);
        mma_bf16_m16n8k16(e[n], al, bh);
      }
    }
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int r = 0; r < 4; ++r) d[n][r] += e[n][r];
    return;
  }
  // the high-high products accumulate in d, the two cross products in e: four independent
  // accumulation chains per call instead of two
  float e[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll 4
  for (int k0 = 0; k0 < K; k0 += 8) {
    const float xv[4] = {x[g * x_si + (k0 + c) * x_sk], x[(g + 8) * x_si + (k0 + c) * x_sk],
                         x[g * x_si + (k0 + c + 4) * x_sk], x[(g + 8) * x_si + (k0 + c + 4) * x_sk]};
    uint32_t xh[4], xl[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      xh[i] = to_tf32(xv[i]);
      xl[i] = to_tf32(xv[i] - __uint_as_float(xh[i]));
    }
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      const float y0 = y[(k0 + c) * y_sk + (g + 8 * n) * y_sj], y1 = y[(k0 + c + 4) * y_sk + (g + 8 * n) * y_sj];
      const uint32_t yh[2] = {to_tf32(y0), to_tf32(y1)};
      const uint32_t yl[2] = {to_tf32(y0 - __uint_as_float(yh[0])), to_tf32(y1 - __uint_as_float(yh[1]))};
      mma_tf32_m16n8k8(d[n], xh, yh);
      if (SPLIT) {
        mma_tf32_m16n8k8(e[n], xh, yl);
        mma_tf32_m16n8k8(e[n], xl, yh);
      }
    }
  }
#pragma unroll
  for (int n = 0; n < 2; ++n)
#pragma unroll
    for (int r = 0; r < 4; ++r) d[n][r] += e[n][r];
}

__device__ __forceinline__ void zero16(float (&d)[2][4]) {
#pragma unroll
  for (int n = 0; n < 2; ++n)
#pragma unroll
    for (int r = 0; r < 4; ++r) d[n][r] = 0.f;
}

// Row / column of fragment element (n, r) inside its 16 x 16 tile.
__device__ __forceinline__ int frow(int lane, int r) { return (lane >> 2) + (r >= 2 ? 8 : 0); }
__device__ __forceinline__ int fcol(int lane, int n, int r) { return 8 * n + 2 * (lane & 3) + (r & 1); }

// T = (I + A)^-1 for the strictly lower A (row stride LD_C): lane = column, forward
// substitution with four partial sums per row (a quarter of the dependency chain).
__device__ __forceinline__ void solve_T(float *Tb, const float *Ab, int lane) {
  float col[kC];
#pragma unroll
  for (int i = 0; i < kC; ++i) {
    float acc[4] = {(i == lane) ? 1.f : 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int k = 0; k < i; ++k) acc[k & 3] = fmaf(-Ab[i * LD_C + k], col[k], acc[k & 3]);
    col[i] = (acc[0] + acc[1]) + (acc[2] + acc[3]);
  }
#pragma unroll
  for (int i = 0; i < kC; ++i) Tb[i * LD_C + lane] = col[i];
}

// Sub-chunk inputs: key / query phasors (and write keys), values, output gradients, gates.
// Rows past n and channels past D / Dv are zero.
template <bool CB>
__device__ void load_sub_chunk(const BwdArgs &a, float *sm, int b, int h, int t0, int n, bool with_q, bool with_do,
                               int64_t row_base) {
  constexpr int kPer = kC * 64 / kBwdThreads;  // elements per thread
  const int tid = threadIdx.x;
  float *gv = sm + O_GV, *br = sm + O_BR, *bi = sm + O_BI;
  // every global load of this thread first, then the arithmetic and the shared stores
  float xk[kPer], xq[kPer], xv[kPer], xo[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int idx = tid + i * kBwdThreads, r = idx >> 6, c = idx & 63, t = t0 + r;
    const bool ok = r < n;
    xk[i] = xq[i] = xv[i] = xo[i] = 0.f;
    if (ok && c < a.D) {
      xk[i] = load_any(a.tk, a.in_dt, b * a.s_tk.b + h * a.s_tk.h + (int64_t)t * a.s_tk.t + c);
      if (with_q) xq[i] = load_any(a.tq, a.in_dt, b * a.s_tq.b + h * a.s_tq.h + (int64_t)t * a.s_tq.t + c);
    }
    if (ok && c < a.Dv) {
      xv[i] = load_any(a.v, a.in_dt, b * a.s_v.b + h * a.s_v.h + (int64_t)t * a.s_v.t + c);
      if (with_do) xo[i] = a.dout[row_base + (int64_t)t * a.Dv + c];
    }
  }
  if (tid < kC) {
    const float g = tid < n ? load_any(a.g, a.g_dt, b * a.s_g.b + h * a.s_g.h + (int64_t)(t0 + tid) * a.s_g.t) : 0.f;
    if (CB) {
      float sp, cp;
      sincosf(g, &sp, &cp);
      br[tid] = tid < n ? 1.f + cp : 0.f;
      bi[tid] = tid < n ? sp : 0.f;
      gv[tid] = tid < n ? 1.f : 0.f;
    } else {
      gv[tid] = g;
    }
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int idx = tid + i * kBwdThreads, r = idx >> 6, c = idx & 63;
    float ck = 0.f, sk = 0.f, cq = 0.f, sq = 0.f;
    if (r < n && c < a.D) {
      sincos_2pi_fast(xk[i], &sk, &ck);
      if (with_q) sincos_2pi_fast(xq[i], &sq, &cq);
    }
    *reinterpret_cast<float2 *>(sm + O_K + r * LD_F + 2 * c) = make_float2(ck, sk);
    if (with_q) *reinterpret_cast<float2 *>(sm + O_Q + r * LD_F + 2 * c) = make_float2(cq, sq);
    if (CB)
      *reinterpret_cast<float2 *>(sm + O_W + r * LD_F + 2 * c) =
          make_float2(fmaf(br[r], ck, -bi[r] * sk), fmaf(br[r], sk, bi[r] * ck));
    sm[O_V + r * LD_V + c] = xv[i];
    if (with_do) sm[O_DO + r * LD_V + c] = xo[i];
  }
}

// State^T (F x Dv, dense in global) <-> shared memory (row stride LD_S), 16-byte accesses,
// all loads of a thread issued before its stores.
__device__ __forceinline__ void state_to_smem(float *dst, const float *src) {
  constexpr int kPer = kF * kDv / 4 / kBwdThreads;
  float4 x[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) x[i] = reinterpret_cast<const float4 *>(src)[threadIdx.x + i * kBwdThreads];
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int q = threadIdx.x + i * kBwdThreads, j = q / (kDv / 4), o4 = q % (kDv / 4);
    *reinterpret_cast<float4 *>(dst + j * LD_S + 4 * o4) = x[i];
  }
}
__device__ __forceinline__ void state_to_global(float *dst, const float *src) {
  constexpr int kPer = kF * kDv / 4 / kBwdThreads;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int q = threadIdx.x + i * kBwdThreads, j = q / (kDv / 4), o4 = q % (kDv / 4);
    reinterpret_cast<float4 *>(dst)[q] = *reinterpret_cast<const float4 *>(src + j * LD_S + 4 * o4);
  }
}

// G = K W^T (C x C) into Gb and A = strict_lower(G) diag(g) / D into the dA buffer (free
// until the dA phase): tiles 0..3 (2 x 2 of 16 x 16).
__device__ __forceinline__ void gram_tile(float *sm, const float *Wb, int tile, float invD, int lane) {
  const int rb = tile >> 1, cb = tile & 1;
  float d[2][4];
  zero16(d);
  mma16<kF>(d, sm + O_K + rb * 16 * LD_F, LD_F, 1, Wb + cb * 16 * LD_F, 1, LD_F, lane);
#pragma unroll
  for (int n = 0; n < 2; ++n)
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int t = rb * 16 + frow(lane, r), s2 = cb * 16 + fcol(lane, n, r);
      sm[O_G + t * LD_C + s2] = d[n][r];
      sm[O_DA + t * LD_C + s2] = s2 < t ? d[n][r] * sm[O_GV + s2] * invD : 0.f;
    }
}

// E = V - K S^T / D (C x Dv) into the dE buffer: tiles 0..7 (2 x 4).
__device__ __forceinline__ void e_tile(float *sm, int tile, float invD, int lane) {
  const int rb = tile >> 2, cb = tile & 3;
  float d[2][4];
  zero16(d);
  mma16<kF>(d, sm + O_K + rb * 16 * LD_F, LD_F, 1, sm + O_ST + cb * 16, LD_S, 1, lane);
#pragma unroll
  for (int n = 0; n < 2; ++n)
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int i = (rb * 16 + frow(lane, r)) * LD_V + cb * 16 + fcol(lane, n, r);
      sm[O_DE + i] = sm[O_V + i] - d[n][r] * invD;
    }
}

// Y = T E (C x Dv) into Yb; with U = diag(g) Y into `u_out` (a C x Dv buffer) when given.
template <bool SPLIT>
__device__ __forceinline__ void y_tile(float *sm, int tile, float *u_out, int lane) {
  const int rb = tile >> 2, cb = tile & 3;
  float d[2][4];
  zero16(d);
  mma16<kC, SPLIT>(d, sm + O_T + rb * 16 * LD_C, LD_C, 1, sm + O_DE + cb * 16, LD_V, 1, lane);
#pragma unroll
  for (int n = 0; n < 2; ++n)
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int row = rb * 16 + frow(lane, r);
      const int i = row * LD_V + cb * 16 + fcol(lane, n, r);
      sm[O_Y + i] = d[n][r];
      if (u_out) u_out[i] = sm[O_GV + row] * d[n][r];
    }
}

template <bool CB>
__global__ void __launch_bounds__(kBwdThreads, 1) core_bwd_kernel(BwdArgs a) {
  extern __shared__ __align__(16) float sm[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.x, b = bh / a.H, h = bh % a.H;
  const int L = a.L, D = a.D, Dv = a.Dv, F = 2 * D;
  const float invD = 1.0f / (float)D;
  const int nsc = (L + kC - 1) / kC;
  const int64_t row_base = (int64_t)bh * L * Dv;
  const int64_t st_base = (int64_t)bh * Dv * F;
  float *ckpt = a.ckpt + (int64_t)bh * nsc * kF * kDv;
  const float *Wb = CB ? sm + O_W : sm + O_K;

  // state^T from the complex state (row o, interleaved column j)
  for (int idx = tid; idx < kF * kDv; idx += kBwdThreads) {
    const int j = idx / kDv, o = idx % kDv;
    sm[O_ST + j * LD_S + o] = (a.state_in && j < F && o < Dv) ? a.state_in[st_base + (int64_t)o * F + j] : 0.f;
  }

  // ---- pass 1: the chunked forward, keeping the state at every sub-chunk start
  for (int sc = 0; sc < nsc; ++sc) {
    const int t0 = sc * kC, n = min(kC, L - t0);
    __syncthreads();
    state_to_global(ckpt + (int64_t)sc * kF * kDv, sm + O_ST);
    load_sub_chunk<CB>(a, sm, b, h, t0, n, false, false, row_base);
    __syncthreads();
    if (warp < 4) gram_tile(sm, Wb, warp, invD, lane);
    __syncthreads();
    if (warp == 0)
      solve_T(sm + O_T, sm + O_DA, lane);
    else
      for (int tile = warp - 1; tile < 8; tile += 7) e_tile(sm, tile, invD, lane);
    __syncthreads();
    y_tile<true>(sm, warp, sm + O_DU, lane);  // U into the dU buffer
    __syncthreads();
    // S^T += W^T U  (F x Dv: 8 x 4 tiles, 4 per warp)
    for (int tile = warp; tile < 32; tile += 8) {
      const int rb = tile >> 2, cb = tile & 3;
      float d[2][4];
#pragma unroll
      for (int nn = 0; nn < 2; ++nn)
#pragma unroll
        for (int r = 0; r < 4; ++r) d[nn][r] = sm[O_ST + (rb * 16 + frow(lane, r)) * LD_S + cb * 16 + fcol(lane, nn, r)];
      mma16<kC>(d, Wb + rb * 16, 1, LD_F, sm + O_DU + cb * 16, LD_V, 1, lane);
#pragma unroll
      for (int nn = 0; nn < 2; ++nn)
#pragma unroll
        for (int r = 0; r < 4; ++r) sm[O_ST + (rb * 16 + frow(lane, r)) * LD_S + cb * 16 + fcol(lane, nn, r)] = d[nn][r];
    }
  }

  // ---- pass 2: backwards over the sub-chunks
  __syncthreads();
  for (int idx = tid; idx < kF * kDv; idx += kBwdThreads) {
    const int j = idx / kDv, o = idx % kDv;
    sm[O_DST + j * LD_S + o] =
        (a.dstate_out && j < F && o < Dv) ? a.dstate_out[st_base + (int64_t)o * F + j] : 0.f;
  }
  for (int sc = nsc - 1; sc >= 0; --sc) {
    const int t0 = sc * kC, n = min(kC, L - t0);
    __syncthreads();
    state_to_smem(sm + O_ST, ckpt + (int64_t)sc * kF * kDv);
    if (tid < kC) sm[O_DG + tid] = 0.f;
    load_sub_chunk<CB>(a, sm, b, h, t0, n, true, true, row_base);
    __syncthreads();
    // G = K W^T (warps 0..3), P = tril(Q W^T) (warps 4..7)
    if (warp < 4) {
      gram_tile(sm, Wb, warp, invD, lane);
    } else {
      const int tile = warp - 4, rb = tile >> 1, cb = tile & 1;
      float d[2][4];
      zero16(d);
      mma16<kF>(d, sm + O_Q + rb * 16 * LD_F, LD_F, 1, Wb + cb * 16 * LD_F, 1, LD_F, lane);
#pragma unroll
      for (int nn = 0; nn < 2; ++nn)
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int t = rb * 16 + frow(lane, r), s = cb * 16 + fcol(lane, nn, r);
          sm[O_P + t * LD_C + s] = s <= t ? d[nn][r] : 0.f;
        }
    }
    __syncthreads();
    // warp 0: T; the others: E and dU = W dS^T + P^T dO / D (neither needs T)
    if (warp == 0) {
      solve_T(sm + O_T, sm + O_DA, lane);
    } else {
      for (int tile = warp - 1; tile < 16; tile += 7) {
        if (tile < 8) {
          e_tile(sm, tile, invD, lane);
        } else {
          const int rb = (tile - 8) >> 2, cb = (tile - 8) & 3;
          float d1[2][4], d2[2][4];
          zero16(d1);
          zero16(d2);
          mma16<kF>(d1, Wb + rb * 16 * LD_F, LD_F, 1, sm + O_DST + cb * 16, LD_S, 1, lane);
          mma16<kC>(d2, sm + O_P + rb * 16, 1, LD_C, sm + O_DO + cb * 16, LD_V, 1, lane);
#pragma unroll
          for (int nn = 0; nn < 2; ++nn)
#pragma unroll
            for (int r = 0; r < 4; ++r)
              sm[O_DU + (rb * 16 + frow(lane, r)) * LD_V + cb * 16 + fcol(lane, nn, r)] = d1[nn][r] + d2[nn][r] * invD;
        }
      }
    }
    __syncthreads();
    y_tile<false>(sm, warp, sm + O_V, lane);  // Y, and U into the V buffer
    __syncthreads();
    // dg += rowsum(dU o Y) (real beta); dY = diag(g) dU in place (a warp per 4 rows)
#pragma unroll
    for (int rr = 0; rr < 4; ++rr) {
      const int row = 4 * warp + rr;
      const float gr = sm[O_GV + row];
      float rs = 0.f;
#pragma unroll
      for (int oo = 0; oo < kDv; oo += 32) {
        const int i = row * LD_V + oo + lane;
        const float du = sm[O_DU + i];
        rs = fmaf(du, sm[O_Y + i], rs);
        sm[O_DU + i] = gr * du;
      }
      if (!CB) {
#pragma unroll
        for (int o2 = 16; o2 >= 1; o2 >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, o2);
        if (lane == 0) sm[O_DG + row] += rs;
      }
    }
    __syncthreads();
    // dE = T^T dY
    {
      const int rb = warp >> 2, cb = warp & 3;
      float d[2][4];
      zero16(d);
      mma16<kC>(d, sm + O_T + rb * 16, 1, LD_C, sm + O_DU + cb * 16, LD_V, 1, lane);
#pragma unroll
      for (int nn = 0; nn < 2; ++nn)
#pragma unroll
        for (int r = 0; r < 4; ++r) sm[O_DE + (rb * 16 + frow(lane, r)) * LD_V + cb * 16 + fcol(lane, nn, r)] = d[nn][r];
    }
    __syncthreads();
    if (warp < 4) {
      // dA = -strict_lower(dE Y^T); dG = dA diag(g) / D; dg += colsum(dA o G) / D
      const int rb = warp >> 1, cb = warp & 1;
      float d[2][4];
      zero16(d);
      mma16<kDv, false>(d, sm + O_DE + rb * 16 * LD_V, LD_V, 1, sm + O_Y + cb * 16 * LD_V, 1, LD_V, lane);
      float cs[2][2] = {{0.f, 0.f}, {0.f, 0.f}};  // [n][col parity]
#pragma unroll
      for (int nn = 0; nn < 2; ++nn)
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int t = rb * 16 + frow(lane, r), s = cb * 16 + fcol(lane, nn, r);
          const float da = s < t ? -d[nn][r] : 0.f;
          sm[O_DA + t * LD_C + s] = da * sm[O_GV + s] * invD;
          cs[nn][r & 1] = fmaf(da, sm[O_G + t * LD_C + s], cs[nn][r & 1]);
        }
      if (!CB) {
#pragma unroll
        for (int nn = 0; nn < 2; ++nn)
#pragma unroll
          for (int p = 0; p < 2; ++p) {
            float v2 = cs[nn][p];
#pragma unroll
            for (int o2 = 4; o2 < 32; o2 <<= 1) v2 += __shfl_xor_sync(0xffffffffu, v2, o2);
            if (lane < 4) atomicAdd(&sm[O_DG + cb * 16 + 8 * nn + 2 * lane + p], v2 * invD);
          }
      }
    } else {
      // dP = tril(dO U^T) / D  (U in the V buffer)
      const int tile = warp - 4, rb = tile >> 1, cb = tile & 1;
      float d[2][4];
      zero16(d);
      mma16<kDv, false>(d, sm + O_DO + rb * 16 * LD_V, LD_V, 1, sm + O_V + cb * 16 * LD_V, 1, LD_V, lane);
#pragma unroll
      for (int nn = 0; nn < 2; ++nn)
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int t = rb * 16 + frow(lane, r), s = cb * 16 + fcol(lane, nn, r);
          sm[O_DP + t * LD_C + s] = s <= t ? d[nn][r] * invD : 0.f;
        }
    }
    __syncthreads();
    // dK, dQ (32 x F: 2 x 8 tiles, 2 per warp) -> d theta_k, d theta_q; dphi (complex beta)
    for (int tile = warp; tile < 16; tile += 8) {
      const int rb = tile >> 3, cb = tile & 7;
      if (cb * 16 >= F) continue;  // columns past 2D (warp-uniform)
      float kr[2][4], ks[2][4], kw[2][4], q1[2][4], q2[2][4];
      zero16(kr);
      zero16(ks);
      zero16(kw);
      zero16(q1);
      zero16(q2);
      // dG W, dG^T K, U dS, dP^T Q, -dE S / D
      mma16<kC, false>(kr, sm + O_DA + rb * 16 * LD_C, LD_C, 1, Wb + cb * 16, LD_F, 1, lane);
      mma16<kC, false>(kw, sm + O_DA + rb * 16, 1, LD_C, sm + O_K + cb * 16, LD_F, 1, lane);
      mma16<kDv, false>(kw, sm + O_V + rb * 16 * LD_V, LD_V, 1, sm + O_DST + cb * 16 * LD_S, 1, LD_S, lane);
      mma16<kC, false>(kw, sm + O_DP + rb * 16, 1, LD_C, sm + O_Q + cb * 16, LD_F, 1, lane);
      mma16<kDv, false>(ks, sm + O_DE + rb * 16 * LD_V, LD_V, 1, sm + O_ST + cb * 16 * LD_S, 1, LD_S, lane);
      // dO S / D, dP W
      mma16<kDv, false>(q1, sm + O_DO + rb * 16 * LD_V, LD_V, 1, sm + O_ST + cb * 16 * LD_S, 1, LD_S, lane);
      mma16<kC, false>(q2, sm + O_DP + rb * 16 * LD_C, LD_C, 1, Wb + cb * 16, LD_F, 1, lane);
      float dphi[2] = {0.f, 0.f};
#pragma unroll
      for (int nn = 0; nn < 2; ++nn)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int t = rb * 16 + frow(lane, 2 * hh), j = cb * 16 + fcol(lane, nn, 0), ch = j >> 1;
          const float kc = sm[O_K + t * LD_F + j], ksn = sm[O_K + t * LD_F + j + 1];
          float dkc = kr[nn][2 * hh] - ks[nn][2 * hh] * invD, dks = kr[nn][2 * hh + 1] - ks[nn][2 * hh + 1] * invD;
          const float dwc = kw[nn][2 * hh], dws = kw[nn][2 * hh + 1];
          if (CB) {
            const float brt = sm[O_BR + t], bit = sm[O_BI + t];
            dkc += brt * dwc + bit * dws;
            dks += -bit * dwc + brt * dws;
            const float dbr = -bit, dbi = brt - 1.f;
            dphi[hh] += dwc * (dbr * kc - dbi * ksn) + dws * (dbr * ksn + dbi * kc);
          } else {
            dkc += dwc;
            dks += dws;
          }
          const float qc = sm[O_Q + t * LD_F + j], qs = sm[O_Q + t * LD_F + j + 1];
          const float dqc = q1[nn][2 * hh] * invD + q2[nn][2 * hh], dqs = q1[nn][2 * hh + 1] * invD + q2[nn][2 * hh + 1];
          if (t < n && ch < D) {
            const int64_t gi = ((int64_t)bh * L + t0 + t) * D + ch;
            a.dtk[gi] = -ksn * dkc + kc * dks;
            a.dtq[gi] = -qs * dqc + qc * dqs;
          }
        }
      if (CB) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          dphi[hh] += __shfl_xor_sync(0xffffffffu, dphi[hh], 1);
          dphi[hh] += __shfl_xor_sync(0xffffffffu, dphi[hh], 2);
        }
        if ((lane & 3) == 0) {
          atomicAdd(&sm[O_DG + rb * 16 + (lane >> 2)], dphi[0]);
          atomicAdd(&sm[O_DG + rb * 16 + (lane >> 2) + 8], dphi[1]);
        }
      }
    }
    __syncthreads();
    // dS^T += Q^T dO / D - K^T dE / D  (F x Dv: 8 x 4 tiles, 4 per warp); dv, dg out
    for (int tile = warp; tile < 32; tile += 8) {
      const int rb = tile >> 2, cb = tile & 3;
      float dq[2][4], dk[2][4];
      zero16(dq);
      zero16(dk);
      mma16<kC>(dq, sm + O_Q + rb * 16, 1, LD_F, sm + O_DO + cb * 16, LD_V, 1, lane);
      mma16<kC>(dk, sm + O_K + rb * 16, 1, LD_F, sm + O_DE + cb * 16, LD_V, 1, lane);
#pragma unroll
      for (int nn = 0; nn < 2; ++nn)
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int i = (rb * 16 + frow(lane, r)) * LD_S + cb * 16 + fcol(lane, nn, r);
          sm[O_DST + i] += (dq[nn][r] - dk[nn][r]) * invD;
        }
    }
    for (int idx = tid; idx < kC * kDv; idx += kBwdThreads) {
      const int r = idx / kDv, o = idx % kDv;
      if (r < n && o < Dv) a.dv[row_base + (int64_t)(t0 + r) * Dv + o] = sm[O_DE + r * LD_V + o];
    }
    if (tid < n) a.dg[(int64_t)bh * L + t0 + tid] = sm[O_DG + tid];
  }
  __syncthreads();
  if (a.dstate_in) {
    for (int idx = tid; idx < Dv * F; idx += kBwdThreads) {
      const int o = idx / F, j = idx % F;
      a.dstate_in[st_base + idx] = sm[O_DST + j * LD_S + o];
    }
  }
}

}  // namespace
}  // namespace dp

extern "C" size_t dp_core_bwd_workspace_size(int B, int H, int L, int Dv) {
  (void)Dv;
  if (B <= 0 || H <= 0 || L <= 0) return 0;
  const size_t nsc = ((size_t)L + dp::kC - 1) / dp::kC;
  return (size_t)B * H * nsc * dp::kF * dp::kDv * sizeof(float);
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
  a.ckpt = static_cast<float *>(workspace);
  a.H = H;
  a.L = L;
  a.D = D;
  a.Dv = Dv;
  auto kern = complex_beta ? core_bwd_kernel<true> : core_bwd_kernel<false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES);
  if (e != cudaSuccess) return set_error(DP_ERR_CUDA, std::string("dp_core_bwd smem attr: ") + cudaGetErrorString(e));
  kern<<<B * H, kBwdThreads, SMEM_BYTES, as_stream(stream)>>>(a);
  return check_launch("core_bwd_kernel");
}
