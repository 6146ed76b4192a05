// Tensor-core (tcgen05) chunkwise complex delta-rule forward for d_k = d_v = 64,
// bf16 inputs, fp32 accumulation.
//
// Reference: _chunkwise_delta_reference (delta_phase/kernels/triton_chunk_delta.py:211-252)
// and the core of DeltaPhaseHolographicBlock.forward (delta_phase/layers.py:203-236).
//
// Real form (see core_simt.cu): per chunk of 64 tokens with key features K (64 x 128,
// interleaved cos/sin), query features Q, values V, write strengths beta and the state
// S (64 x 128, fp32, kept transposed in tensor memory for the whole sequence):
//   G1:  [K; Q] K^T           -> K K^T (Gram) and Q K^T            (TMEM, fp32)
//        A = strict_lower(K K^T / 64) diag(beta);  T = (I + A)^-1  (CUDA cores, fp32)
//   G2:  [bT; P] [K | V]      -> bT K and bT V,   bT = diag(beta) T,  P = tril(Q K^T)
//   G3:  [W; Q] S^T           -> W S^T, Q S^T,    W = bT K
//        U = bT V - W S^T / 64                                    (the delta-rule writes)
//   G4:  S^T += K^T U         (state update, accumulated in TMEM)
//   G5:  Q S^T += P U   ->  64 * output rows of the chunk
// All five products are tcgen05.mma (kind::f16, bf16 operands from shared memory,
// fp32 accumulators in tensor memory) issued by one thread.  Operand tiles use the
// SWIZZLE_NONE core-matrix layout (8 rows x 16 bytes per core matrix), so the same
// buffer serves as a K-major or MN-major operand by swapping the two stride fields:
// K is read as A (G1), B (G1), B (G2) and A^T (G4) without copies.
//
// One CTA of 128 threads per (batch, head); inputs stream in with bulk async copies
// (cp.async.bulk + mbarrier, two stages ahead); every wait is bounded.
#include "dp_common.cuh"
#include "tc_ptx.cuh"

namespace dp {

int *device_error_ptr();

namespace {

using namespace ptx;

constexpr int kC = 64;     // tokens per chunk
constexpr int kF = 128;    // key features (2 * d_k)
constexpr int kDv = 64;    // value channels
constexpr int kThreads = 128;
constexpr uint64_t kTimeoutNs = 2000000000ull;  // 2 s per wait

// shared-memory map (bytes)
constexpr int RG_KVQ = 24 * 128;                 // row group: 16 feature groups + 8 value groups
constexpr int OFF_KVQ = 0;                       // [K | V] rows 0..63, [Q] rows 64..127
constexpr int OFF_WQ = OFF_KVQ + 16 * RG_KVQ;    // [W; Q], 128 x 128
constexpr int RG_WQ = 16 * 128;
constexpr int OFF_TP = OFF_WQ + 16 * RG_WQ;      // [bT; P], 128 x 64
constexpr int RG_64 = 8 * 128;
constexpr int OFF_U = OFF_TP + 16 * RG_64;       // U, 64 x 64
constexpr int OFF_S0 = OFF_U + 8 * RG_64;        // S^T bf16, 128 x 64
constexpr int OFF_STAGE = OFF_S0 + 16 * RG_64;   // 2 x {theta_k, theta_q, v} raw rows
constexpr int STAGE_BYTES = 3 * kC * 128;
constexpr int OFF_AF = OFF_STAGE + 2 * STAGE_BYTES;  // A (64 x 64 fp32)
constexpr int OFF_BETA = OFF_AF + kC * kC * 4;
constexpr int OFF_BAR = OFF_BETA + kC * 4;
constexpr int SMEM_BYTES = OFF_BAR + 64;

// tensor-memory columns
constexpr uint32_t COL_S = 0, COL_D1 = 64, COL_D2 = 128, COL_DC = 320, TMEM_COLS = 512;

__device__ __forceinline__ uint32_t cm_off(int r, int k, int rg) {
  return (uint32_t)((r >> 3) * rg + (k >> 3) * 128 + (r & 7) * 16 + (k & 7) * 2);
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&h);
}

// sin/cos of a phase: reduce to [-pi, pi] (x - 2 pi round(x / 2 pi), 2 pi split in two
// parts), then the hardware approximation; far below bf16 resolution.
__device__ __forceinline__ void fast_sincos(float x, float *s, float *c) {
  const float k = rintf(x * 0.15915494309189535f);
  float r = fmaf(-k, 6.28318548202514648f, x);
  r = fmaf(-k, -1.7484556e-07f, r);
  __sincosf(r, s, c);
}

__device__ __forceinline__ float load_beta(const void *p, int dt, int64_t i) {
  if (dt == DP_F32) return static_cast<const float *>(p)[i];
  if (dt == DP_BF16) return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
  return __half2float(static_cast<const __half *>(p)[i]);
}

struct TcArgs {
  const __nv_bfloat16 *tk, *tq, *v;
  const void *beta;
  int beta_dt;
  const float *state_in;
  float *out;
  float *state_out;
  int H, L;
  SeqStrides s_tk, s_tq, s_v, s_b, s_out;
  int *err;
};

// Issue the bulk copies of chunk `c0` (rows [c0, c0 + n)) of one (b, h) into a stage.
// Executed by one full warp; lane 0 registers the expected bytes first.
__device__ __forceinline__ void issue_chunk_loads(const TcArgs &a, int b, int h, int c0, int n,
                                                  uint8_t *stage, uint64_t *bar, int lane) {
  if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t)(3 * n * 128));
  __syncwarp();
  const __nv_bfloat16 *src[3] = {a.tk + b * a.s_tk.b + h * a.s_tk.h + (int64_t)c0 * a.s_tk.t,
                                 a.tq + b * a.s_tq.b + h * a.s_tq.h + (int64_t)c0 * a.s_tq.t,
                                 a.v + b * a.s_v.b + h * a.s_v.h + (int64_t)c0 * a.s_v.t};
  const int64_t st[3] = {a.s_tk.t, a.s_tq.t, a.s_v.t};
#pragma unroll
  for (int x = 0; x < 3; ++x) {
    uint8_t *dst = stage + x * kC * 128;
    if (st[x] == 64) {
      if (lane == 0) bulk_g2s(dst, src[x], (uint32_t)(n * 128), bar);
    } else {
      for (int t = lane; t < n; t += 32) bulk_g2s(dst + t * 128, src[x] + t * st[x], 128u, bar);
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1) core_tc_kernel(TcArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t *kvq = smem + OFF_KVQ;
  uint8_t *wq = smem + OFF_WQ;
  uint8_t *tp = smem + OFF_TP;
  uint8_t *ub = smem + OFF_U;
  uint8_t *s0 = smem + OFF_S0;
  float *af = reinterpret_cast<float *>(smem + OFF_AF);
  float *bs = reinterpret_cast<float *>(smem + OFF_BETA);
  uint64_t *mma_bar = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
  uint64_t *load_bar = mma_bar + 1;  // [2]
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_bar + 3);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.x, b = bh / a.H, h = bh % a.H;
  const int L = a.L;
  const int nchunks = (L + kC - 1) / kC;

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
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;

  // prefetch the first two chunks
  if (warp == 3) {
    for (int c = 0; c < 2 && c < nchunks; ++c) {
      const int n = min(kC, L - c * kC);
      issue_chunk_loads(a, b, h, c * kC, n, smem + OFF_STAGE + c * STAGE_BYTES, &load_bar[c], lane);
    }
  }

  // state^T (feature j = lane row, value channel o = column) -> TMEM
  {
    const int j = warp * 32 + lane;
    const int64_t base = (int64_t)bh * kDv * kF;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float vals[16];
#pragma unroll
      for (int i = 0; i < 16; ++i)
        vals[i] = a.state_in ? a.state_in[base + (int64_t)(16 * q + i) * kF + j] : 0.f;
      tmem_st16(tmem + lane_base + COL_S + 16 * q, vals);
    }
    tmem_st_wait();
  }
  tc_fence_before();
  __syncthreads();

  uint32_t mma_phase = 0;
  bool failed = false, mma_pending = false;
  int issued = min(nchunks, 2), consumed = 0;  // chunk loads issued / waited for (uniform)
  const float inv64 = 1.0f / 64.0f;

  for (int c = 0; c < nchunks && !failed; ++c) {
    const int t0 = c * kC;
    const int nvalid = min(kC, L - t0);
    const int st = c & 1;
    uint8_t *stage = smem + OFF_STAGE + st * STAGE_BYTES;

    // ---- phase 0: inputs of this chunk
    bool ok = mbar_wait(&load_bar[st], (uint32_t)((c >> 1) & 1), kTimeoutNs);
    if (__syncthreads_or(!ok)) { failed = true; break; }
    consumed = c + 1;

    // ---- phase 1: phasors (bf16) into the operand tiles, values, beta
    {
      const int t = tid >> 1, hh = tid & 1;
      const bool valid = t < nvalid;
      const __nv_bfloat16 *rk = reinterpret_cast<const __nv_bfloat16 *>(stage + t * 128);
      const __nv_bfloat16 *rq = reinterpret_cast<const __nv_bfloat16 *>(stage + kC * 128 + t * 128);
#pragma unroll 2
      for (int gg = 0; gg < 8; ++gg) {
        const int g = 8 * hh + gg;  // feature group: channels 4g .. 4g+3
        uint4 kw = make_uint4(0, 0, 0, 0), qw = make_uint4(0, 0, 0, 0);
        if (valid) {
          float s0_, c0_, s1_, c1_, s2_, c2_, s3_, c3_;
          const uint2 kraw = *reinterpret_cast<const uint2 *>(rk + 4 * g);
          const __nv_bfloat162 k01 = *reinterpret_cast<const __nv_bfloat162 *>(&kraw.x);
          const __nv_bfloat162 k23 = *reinterpret_cast<const __nv_bfloat162 *>(&kraw.y);
          fast_sincos(__low2float(k01), &s0_, &c0_);
          fast_sincos(__high2float(k01), &s1_, &c1_);
          fast_sincos(__low2float(k23), &s2_, &c2_);
          fast_sincos(__high2float(k23), &s3_, &c3_);
          kw = make_uint4(pack_bf16(c0_, s0_), pack_bf16(c1_, s1_), pack_bf16(c2_, s2_), pack_bf16(c3_, s3_));
          const uint2 qraw = *reinterpret_cast<const uint2 *>(rq + 4 * g);
          const __nv_bfloat162 q01 = *reinterpret_cast<const __nv_bfloat162 *>(&qraw.x);
          const __nv_bfloat162 q23 = *reinterpret_cast<const __nv_bfloat162 *>(&qraw.y);
          fast_sincos(__low2float(q01), &s0_, &c0_);
          fast_sincos(__high2float(q01), &s1_, &c1_);
          fast_sincos(__low2float(q23), &s2_, &c2_);
          fast_sincos(__high2float(q23), &s3_, &c3_);
          qw = make_uint4(pack_bf16(c0_, s0_), pack_bf16(c1_, s1_), pack_bf16(c2_, s2_), pack_bf16(c3_, s3_));
        }
        *reinterpret_cast<uint4 *>(kvq + cm_off(t, 8 * g, RG_KVQ)) = kw;
        *reinterpret_cast<uint4 *>(kvq + cm_off(64 + t, 8 * g, RG_KVQ)) = qw;
        *reinterpret_cast<uint4 *>(wq + cm_off(64 + t, 8 * g, RG_WQ)) = qw;
      }
      const uint8_t *rv = stage + 2 * kC * 128 + t * 128;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int vg = 4 * hh + i;  // value channels 8 vg .. 8 vg + 7
        uint4 w = valid ? *reinterpret_cast<const uint4 *>(rv + vg * 16) : make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4 *>(kvq + cm_off(t, 128 + 8 * vg, RG_KVQ)) = w;
      }
      if (tid < kC)
        bs[tid] = (tid < nvalid)
                      ? load_beta(a.beta, a.beta_dt,
                                  b * a.s_b.b + h * a.s_b.h + (int64_t)(t0 + tid) * a.s_b.t)
                      : 0.f;
    }
    fence_proxy_async_smem();
    __syncthreads();

    // ---- phase 2: stage `st` is free again -> prefetch chunk c+2; G1 = [K; Q] K^T
    if (c + 2 < nchunks) {
      if (warp == 3) {
        const int n = min(kC, L - (c + 2) * kC);
        issue_chunk_loads(a, b, h, (c + 2) * kC, n, stage, &load_bar[st], lane);
      }
      issued = c + 3;
    }
    if (tid == 0) {
      tc_fence_after();
      const uint32_t sa = smem_u32(kvq);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        mma_f16_ss(tmem + COL_D1, make_desc(sa + kk * 256, 128, RG_KVQ),
                   make_desc(sa + kk * 256, 128, RG_KVQ), idesc_bf16(128, 64, false, false), kk > 0);
      mma_commit(mma_bar);
    }
    ok = mbar_wait(mma_bar, mma_phase, kTimeoutNs);
    mma_phase ^= 1;
    if (__syncthreads_or(!ok)) { failed = mma_pending = true; break; }
    tc_fence_after();

    // ---- phase 3: A (fp32, rows 0..63) and P = tril(Q K^T) (bf16, rows 64..127 of TP)
    {
      const int row = warp * 32 + lane;  // TMEM lane
      if (warp < 2) {
        const int t = row;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float g[16];
          tmem_ld16(tmem + lane_base + COL_D1 + 16 * q, g);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; i += 4) {
            const int s = 16 * q + i;
            float4 w;
            w.x = (s + 0 < t) ? g[i + 0] * inv64 * bs[s + 0] : 0.f;
            w.y = (s + 1 < t) ? g[i + 1] * inv64 * bs[s + 1] : 0.f;
            w.z = (s + 2 < t) ? g[i + 2] * inv64 * bs[s + 2] : 0.f;
            w.w = (s + 3 < t) ? g[i + 3] * inv64 * bs[s + 3] : 0.f;
            *reinterpret_cast<float4 *>(af + t * kC + s) = w;
          }
        }
      } else {
        const int t = row - 64;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float p[16];
          tmem_ld16(tmem + lane_base + COL_D1 + 16 * q, p);
          tmem_ld_wait();
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            const int s = 16 * q + 8 * half;
            uint4 w;
            w.x = pack_bf16(s + 0 <= t ? p[8 * half + 0] : 0.f, s + 1 <= t ? p[8 * half + 1] : 0.f);
            w.y = pack_bf16(s + 2 <= t ? p[8 * half + 2] : 0.f, s + 3 <= t ? p[8 * half + 3] : 0.f);
            w.z = pack_bf16(s + 4 <= t ? p[8 * half + 4] : 0.f, s + 5 <= t ? p[8 * half + 5] : 0.f);
            w.w = pack_bf16(s + 6 <= t ? p[8 * half + 6] : 0.f, s + 7 <= t ? p[8 * half + 7] : 0.f);
            *reinterpret_cast<uint4 *>(tp + cm_off(64 + t, s, RG_64)) = w;
          }
        }
      }
    }
    tc_fence_before();
    __syncthreads();

    // ---- phase 4: T = (I + A)^-1 by forward substitution (thread j owns column j);
    //      bT = diag(beta) T -> rows 0..63 of TP
    if (tid < kC) {
      const int j = tid;
      float col[kC];
#pragma unroll
      for (int i = 0; i < kC; ++i) {
        float acc0 = (i == j) ? 1.f : 0.f, acc1 = 0.f;
        const float *ar = af + i * kC;
#pragma unroll
        for (int k = 0; k + 1 < i; k += 2) {
          acc0 = fmaf(-ar[k], col[k], acc0);
          acc1 = fmaf(-ar[k + 1], col[k + 1], acc1);
        }
        if (i & 1) acc0 = fmaf(-ar[i - 1], col[i - 1], acc0);
        col[i] = acc0 + acc1;
      }
#pragma unroll
      for (int i = 0; i < kC; ++i)
        *reinterpret_cast<__nv_bfloat16 *>(tp + cm_off(i, j, RG_64)) = __float2bfloat16_rn(bs[i] * col[i]);
    }
    fence_proxy_async_smem();
    __syncthreads();

    // ---- phase 5: G2 = [bT; P] [K | V]  (N = 192)
    if (tid == 0) {
      tc_fence_after();
      const uint32_t sa = smem_u32(tp), sb = smem_u32(kvq);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        mma_f16_ss(tmem + COL_D2, make_desc(sa + kk * 256, 128, RG_64),
                   make_desc(sb + kk * 2 * RG_KVQ, RG_KVQ, 128), idesc_bf16(128, 192, false, true),
                   kk > 0);
      mma_commit(mma_bar);
    }
    ok = mbar_wait(mma_bar, mma_phase, kTimeoutNs);
    mma_phase ^= 1;
    if (__syncthreads_or(!ok)) { failed = mma_pending = true; break; }
    tc_fence_after();

    // ---- phase 6: W = bT K (bf16, rows 0..63 of WQ), keep bT V in registers; S^T -> bf16
    float ut[64];
    if (warp < 2) {
      const int t = warp * 32 + lane;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float w[16];
        tmem_ld16(tmem + lane_base + COL_D2 + 16 * q, w);
        tmem_ld_wait();
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint4 pk;
          pk.x = pack_bf16(w[8 * half + 0], w[8 * half + 1]);
          pk.y = pack_bf16(w[8 * half + 2], w[8 * half + 3]);
          pk.z = pack_bf16(w[8 * half + 4], w[8 * half + 5]);
          pk.w = pack_bf16(w[8 * half + 6], w[8 * half + 7]);
          *reinterpret_cast<uint4 *>(wq + cm_off(t, 16 * q + 8 * half, RG_WQ)) = pk;
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float w[16];
        tmem_ld16(tmem + lane_base + COL_D2 + 128 + 16 * q, w);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) ut[16 * q + i] = w[i];
      }
    }
    {
      const int j = warp * 32 + lane;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float sv[16];
        tmem_ld16(tmem + lane_base + COL_S + 16 * q, sv);
        tmem_ld_wait();
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint4 pk;
          pk.x = pack_bf16(sv[8 * half + 0], sv[8 * half + 1]);
          pk.y = pack_bf16(sv[8 * half + 2], sv[8 * half + 3]);
          pk.z = pack_bf16(sv[8 * half + 4], sv[8 * half + 5]);
          pk.w = pack_bf16(sv[8 * half + 6], sv[8 * half + 7]);
          *reinterpret_cast<uint4 *>(s0 + cm_off(j, 16 * q + 8 * half, RG_64)) = pk;
        }
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();

    // ---- phase 7: G3 = [W; Q] S^T
    if (tid == 0) {
      tc_fence_after();
      const uint32_t sa = smem_u32(wq), sb = smem_u32(s0);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        mma_f16_ss(tmem + COL_DC, make_desc(sa + kk * 256, 128, RG_WQ),
                   make_desc(sb + kk * 2 * RG_64, RG_64, 128), idesc_bf16(128, 64, false, true), kk > 0);
      mma_commit(mma_bar);
    }
    ok = mbar_wait(mma_bar, mma_phase, kTimeoutNs);
    mma_phase ^= 1;
    if (__syncthreads_or(!ok)) { failed = mma_pending = true; break; }
    tc_fence_after();

    // ---- phase 8: U = bT V - W S^T / 64 (bf16, for G4 / G5)
    if (warp < 2) {
      const int t = warp * 32 + lane;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float ws[16];
        tmem_ld16(tmem + lane_base + COL_DC + 16 * q, ws);
        tmem_ld_wait();
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int o = 16 * q + 8 * half;
          uint4 pk;
          pk.x = pack_bf16(ut[o + 0] - ws[8 * half + 0] * inv64, ut[o + 1] - ws[8 * half + 1] * inv64);
          pk.y = pack_bf16(ut[o + 2] - ws[8 * half + 2] * inv64, ut[o + 3] - ws[8 * half + 3] * inv64);
          pk.z = pack_bf16(ut[o + 4] - ws[8 * half + 4] * inv64, ut[o + 5] - ws[8 * half + 5] * inv64);
          pk.w = pack_bf16(ut[o + 6] - ws[8 * half + 6] * inv64, ut[o + 7] - ws[8 * half + 7] * inv64);
          *reinterpret_cast<uint4 *>(ub + cm_off(t, o, RG_64)) = pk;
        }
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();

    // ---- phase 9: G4  S^T += K^T U ;  G5  D_C += [bT; P] U  (rows 64..127 become 64 O)
    if (tid == 0) {
      tc_fence_after();
      const uint32_t sk = smem_u32(kvq), su = smem_u32(ub), stp = smem_u32(tp);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        mma_f16_ss(tmem + COL_S, make_desc(sk + kk * 2 * RG_KVQ, RG_KVQ, 128),
                   make_desc(su + kk * 2 * RG_64, RG_64, 128), idesc_bf16(128, 64, true, true), 1u);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        mma_f16_ss(tmem + COL_DC, make_desc(stp + kk * 256, 128, RG_64),
                   make_desc(su + kk * 2 * RG_64, RG_64, 128), idesc_bf16(128, 64, false, true), 1u);
      mma_commit(mma_bar);
    }
    ok = mbar_wait(mma_bar, mma_phase, kTimeoutNs);
    mma_phase ^= 1;
    if (__syncthreads_or(!ok)) { failed = mma_pending = true; break; }
    tc_fence_after();

    // ---- phase 10: outputs (rows 64..127 of D_C) / 64 -> global fp32
    if (warp >= 2) {
      const int t = warp * 32 + lane - 64;
      float *orow = a.out + b * a.s_out.b + h * a.s_out.h + (int64_t)(t0 + t) * a.s_out.t;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float o[16];
        tmem_ld16(tmem + lane_base + COL_DC + 16 * q, o);
        tmem_ld_wait();
        if (t < nvalid) {
#pragma unroll
          for (int i = 0; i < 16; i += 4)
            *reinterpret_cast<float4 *>(orow + 16 * q + i) =
                make_float4(o[i] * inv64, o[i + 1] * inv64, o[i + 2] * inv64, o[i + 3] * inv64);
        }
      }
    }
    tc_fence_before();
    __syncthreads();
  }

  if (failed) {
    if (tid == 0) atomicCAS(a.err, 0, DP_ERR_TIMEOUT);
    // let copies and MMAs still in flight land before the shared / tensor memory is
    // released (each wait bounded again)
    for (int k = consumed; k < issued; ++k) mbar_wait(&load_bar[k & 1], (uint32_t)((k >> 1) & 1), kTimeoutNs);
    if (mma_pending) mbar_wait(mma_bar, mma_phase ^ 1, kTimeoutNs);
  } else {
    // final state: TMEM S^T -> complex64 state (row o, interleaved column j)
    tc_fence_after();
    const int j = warp * 32 + lane;
    const int64_t base = (int64_t)bh * kDv * kF;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float sv[16];
      tmem_ld16(tmem + lane_base + COL_S + 16 * q, sv);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 16; ++i) a.state_out[base + (int64_t)(16 * q + i) * kF + j] = sv[i];
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, TMEM_COLS);
}

}  // namespace

// True if dp_core_fwd's arguments fit the tensor-core kernel.
bool core_tc_supported(const void *tk, const void *tq, const void *v, int in_dt, const float *out,
                       int D, int Dv, const SeqStrides *s) {
  if (in_dt != DP_BF16 || D != 64 || Dv != 64) return false;
  auto al16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!al16(tk) || !al16(tq) || !al16(v) || !al16(out)) return false;
  for (int i = 0; i < 3; ++i)
    if ((s[i].b % 8) || (s[i].h % 8) || (s[i].t % 8)) return false;
  if ((s[4].b % 4) || (s[4].h % 4) || (s[4].t % 4)) return false;
  return true;
}

int core_fwd_tc(const void *tk, const void *tq, const void *v, const void *beta, int beta_dt,
                const float *state_in, float *out, float *state_out, int B, int H, int L,
                const SeqStrides *s, cudaStream_t stream) {
  TcArgs a;
  a.tk = static_cast<const __nv_bfloat16 *>(tk);
  a.tq = static_cast<const __nv_bfloat16 *>(tq);
  a.v = static_cast<const __nv_bfloat16 *>(v);
  a.beta = beta;
  a.beta_dt = beta_dt;
  a.state_in = state_in;
  a.out = out;
  a.state_out = state_out;
  a.H = H;
  a.L = L;
  a.s_tk = s[0];
  a.s_tq = s[1];
  a.s_v = s[2];
  a.s_b = s[3];
  a.s_out = s[4];
  a.err = device_error_ptr();
  if (!a.err) return set_error(DP_ERR_CUDA, "core_fwd_tc: device error word unavailable");
  cudaError_t e = cudaFuncSetAttribute(core_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  if (e != cudaSuccess) return set_error(DP_ERR_CUDA, std::string("core_tc smem attr: ") + cudaGetErrorString(e));
  core_tc_kernel<<<B * H, kThreads, SMEM_BYTES, stream>>>(a);
  return check_launch("core_tc_kernel");
}

}  // namespace dp
