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
constexpr int LDA = 68;                              // padded fp32 row stride (bank spread)
constexpr int OFF_AT = OFF_STAGE + 2 * STAGE_BYTES;  // A^T (64 x 64 fp32): At[k][i] = A[i][k]
constexpr int OFF_TF = OFF_AT + kC * LDA * 4;        // T = (I + A)^-1, fp32, diagonal blocks
constexpr int LDY = 36;
constexpr int OFF_Y = OFF_TF + kC * LDA * 4;         // Y = A[32:, :32] T[:32, :32] (32 x 32)
constexpr int OFF_BETA = OFF_Y + 32 * LDY * 4;
constexpr int OFF_BAR = OFF_BETA + 2 * kC * 4;  // beta: two chunk slots
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
// parts), then the hardware approximation; the error is far below bf16 resolution.
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
  float *at = reinterpret_cast<float *>(smem + OFF_AT);
  float *tf = reinterpret_cast<float *>(smem + OFF_TF);
  float *ys = reinterpret_cast<float *>(smem + OFF_Y);
  float *bs2 = reinterpret_cast<float *>(smem + OFF_BETA);
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

  // the upper-right 32 x 32 block of bT (rows 0..31, columns 32..63 of TP) is zero
  for (int i = tid; i < 32 * 4; i += kThreads)
    *reinterpret_cast<uint4 *>(tp + cm_off(i >> 2, 32 + 8 * (i & 3), RG_64)) = make_uint4(0, 0, 0, 0);

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

  // beta of chunk 0 (later chunks are prefetched one chunk ahead)
  if (tid < kC)
    bs2[tid] = (tid < L) ? load_beta(a.beta, a.beta_dt, b * a.s_b.b + h * a.s_b.h + (int64_t)tid * a.s_b.t) : 0.f;
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
    float *bs = bs2 + st * kC;

    // ---- phase 0: inputs of this chunk
    bool ok = mbar_wait(&load_bar[st], (uint32_t)((c >> 1) & 1), kTimeoutNs);
    if (__syncthreads_or(!ok)) { failed = true; break; }
    consumed = c + 1;

    // ---- phase 1: phasors (bf16) into the operand tiles, values, beta.  Work item
    //      p = tid + 128 r covers token row p / 8 and channels 8 (p % 8) .. + 7, so a
    //      warp reads 512 contiguous bytes of the staged rows per step.
    {
      // beta of the next chunk: issue the load now, store it after the phasor work
      float bnext = 0.f;
      if (tid < kC && t0 + kC + tid < L)
        bnext = load_beta(a.beta, a.beta_dt, b * a.s_b.b + h * a.s_b.h + (int64_t)(t0 + kC + tid) * a.s_b.t);
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int p = tid + kThreads * r;
        const int t = p >> 3, sg = p & 7;
        uint4 kraw = make_uint4(0, 0, 0, 0), qraw = kraw, vraw = kraw;
        const bool valid = t < nvalid;
        if (valid) {
          kraw = *reinterpret_cast<const uint4 *>(stage + t * 128 + sg * 16);
          qraw = *reinterpret_cast<const uint4 *>(stage + kC * 128 + t * 128 + sg * 16);
          vraw = *reinterpret_cast<const uint4 *>(stage + 2 * kC * 128 + t * 128 + sg * 16);
        }
        const uint32_t kr[4] = {kraw.x, kraw.y, kraw.z, kraw.w};
        const uint32_t qr[4] = {qraw.x, qraw.y, qraw.z, qraw.w};
        uint32_t kw[8], qw[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float s0_, c0_, s1_, c1_;
          const __nv_bfloat162 kk2 = *reinterpret_cast<const __nv_bfloat162 *>(&kr[i]);
          fast_sincos(__low2float(kk2), &s0_, &c0_);
          fast_sincos(__high2float(kk2), &s1_, &c1_);
          kw[2 * i] = pack_bf16(c0_, s0_);
          kw[2 * i + 1] = pack_bf16(c1_, s1_);
          const __nv_bfloat162 qq2 = *reinterpret_cast<const __nv_bfloat162 *>(&qr[i]);
          fast_sincos(__low2float(qq2), &s0_, &c0_);
          fast_sincos(__high2float(qq2), &s1_, &c1_);
          qw[2 * i] = pack_bf16(c0_, s0_);
          qw[2 * i + 1] = pack_bf16(c1_, s1_);
        }
        if (!valid) {
#pragma unroll
          for (int i = 0; i < 8; ++i) kw[i] = qw[i] = 0u;
        }
        // channels 8 sg .. 8 sg + 7 -> features 16 sg .. 16 sg + 15 (two core-matrix columns)
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const uint4 kv = make_uint4(kw[4 * half], kw[4 * half + 1], kw[4 * half + 2], kw[4 * half + 3]);
          const uint4 qv = make_uint4(qw[4 * half], qw[4 * half + 1], qw[4 * half + 2], qw[4 * half + 3]);
          *reinterpret_cast<uint4 *>(kvq + cm_off(t, 16 * sg + 8 * half, RG_KVQ)) = kv;
          *reinterpret_cast<uint4 *>(kvq + cm_off(64 + t, 16 * sg + 8 * half, RG_KVQ)) = qv;
          *reinterpret_cast<uint4 *>(wq + cm_off(64 + t, 16 * sg + 8 * half, RG_WQ)) = qv;
        }
        *reinterpret_cast<uint4 *>(kvq + cm_off(t, 128 + 8 * sg, RG_KVQ)) = vraw;
      }
      if (tid < kC) bs2[(st ^ 1) * kC + tid] = bnext;
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

    // ---- phase 3: A^T from the (exactly symmetric) Gram rows:  At[k][i] = beta_k G[k][i] / 64
    //      for i > k (row k of TMEM is thread k of warps 0, 1)
    if (warp < 2) {
      const int k = warp * 32 + lane;
      const float bk = bs[k] * inv64;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float g[16];
        tmem_ld16(tmem + lane_base + COL_D1 + 16 * q, g);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; i += 4) {
          const int c0 = 16 * q + i;
          float4 w;
          w.x = (c0 + 0 > k) ? g[i + 0] * bk : 0.f;
          w.y = (c0 + 1 > k) ? g[i + 1] * bk : 0.f;
          w.z = (c0 + 2 > k) ? g[i + 2] * bk : 0.f;
          w.w = (c0 + 3 > k) ? g[i + 3] * bk : 0.f;
          *reinterpret_cast<float4 *>(at + k * LDA + c0) = w;
        }
      }
    }
    tc_fence_before();
    __syncthreads();

    // ---- phase 4a: warps 0, 1 invert the 32 x 32 diagonal blocks of (I + A) by
    //      right-looking substitution (lane = column, the column lives in registers);
    //      warps 2, 3 meanwhile convert P = tril(Q K^T) to bf16 (rows 64..127 of TP).
    if (warp < 2) {
      const int o = warp * 32;  // block offset
      float col[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) col[i] = (i == lane) ? 1.f : 0.f;
#pragma unroll
      for (int k = 0; k < 31; ++k) {
        const float tk = col[k];
        const float *ak = at + (o + k) * LDA + o;  // At[o+k][o+i] = A[o+i][o+k]
#pragma unroll
        for (int i4 = ((k + 1) & ~3); i4 < 32; i4 += 4) {
          const float4 av = *reinterpret_cast<const float4 *>(ak + i4);
          if (i4 + 0 > k) col[i4 + 0] = fmaf(-av.x, tk, col[i4 + 0]);
          if (i4 + 1 > k) col[i4 + 1] = fmaf(-av.y, tk, col[i4 + 1]);
          if (i4 + 2 > k) col[i4 + 2] = fmaf(-av.z, tk, col[i4 + 2]);
          if (i4 + 3 > k) col[i4 + 3] = fmaf(-av.w, tk, col[i4 + 3]);
        }
      }
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        tf[(o + i) * LDA + o + lane] = col[i];
        *reinterpret_cast<__nv_bfloat16 *>(tp + cm_off(o + i, o + lane, RG_64)) =
            __float2bfloat16_rn(bs[o + i] * col[i]);
      }
    } else {
      const int t = warp * 32 + lane - 64;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float p[16];
        tmem_ld16(tmem + lane_base + COL_D1 + 16 * q, p);
        tmem_ld_wait();
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int sidx = 16 * q + 8 * half;
          uint4 w;
          w.x = pack_bf16(sidx + 0 <= t ? p[8 * half + 0] : 0.f, sidx + 1 <= t ? p[8 * half + 1] : 0.f);
          w.y = pack_bf16(sidx + 2 <= t ? p[8 * half + 2] : 0.f, sidx + 3 <= t ? p[8 * half + 3] : 0.f);
          w.z = pack_bf16(sidx + 4 <= t ? p[8 * half + 4] : 0.f, sidx + 5 <= t ? p[8 * half + 5] : 0.f);
          w.w = pack_bf16(sidx + 6 <= t ? p[8 * half + 6] : 0.f, sidx + 7 <= t ? p[8 * half + 7] : 0.f);
          *reinterpret_cast<uint4 *>(tp + cm_off(64 + t, sidx, RG_64)) = w;
        }
      }
    }
    tc_fence_before();
    __syncthreads();

    // ---- phase 4b: Y = A[32:64, 0:32] T00   (thread: column j, rows 8 ib .. 8 ib + 7)
    {
      const int j = lane, ib = warp;
      float y[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll 8
      for (int k = 0; k < 32; ++k) {
        const float tkj = tf[k * LDA + j];
        const float4 a0 = *reinterpret_cast<const float4 *>(at + k * LDA + 32 + 8 * ib);
        const float4 a1 = *reinterpret_cast<const float4 *>(at + k * LDA + 36 + 8 * ib);
        y[0] = fmaf(a0.x, tkj, y[0]); y[1] = fmaf(a0.y, tkj, y[1]);
        y[2] = fmaf(a0.z, tkj, y[2]); y[3] = fmaf(a0.w, tkj, y[3]);
        y[4] = fmaf(a1.x, tkj, y[4]); y[5] = fmaf(a1.y, tkj, y[5]);
        y[6] = fmaf(a1.z, tkj, y[6]); y[7] = fmaf(a1.w, tkj, y[7]);
      }
#pragma unroll
      for (int r = 0; r < 8; ++r) ys[(8 * ib + r) * LDY + j] = y[r];
    }
    __syncthreads();

    // ---- phase 4c: T[32:64, 0:32] = -T11 Y, scaled by beta -> bf16 rows 32..63 of TP
    {
      const int j = lane, ib = warp;
      float x[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll 4
      for (int m = 0; m < 32; m += 4) {
        const float y0 = ys[(m + 0) * LDY + j], y1 = ys[(m + 1) * LDY + j];
        const float y2 = ys[(m + 2) * LDY + j], y3 = ys[(m + 3) * LDY + j];
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          const float4 t4 = *reinterpret_cast<const float4 *>(tf + (32 + 8 * ib + r) * LDA + 32 + m);
          x[r] = fmaf(t4.x, y0, x[r]);
          x[r] = fmaf(t4.y, y1, x[r]);
          x[r] = fmaf(t4.z, y2, x[r]);
          x[r] = fmaf(t4.w, y3, x[r]);
        }
      }
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const int i = 32 + 8 * ib + r;
        *reinterpret_cast<__nv_bfloat16 *>(tp + cm_off(i, j, RG_64)) = __float2bfloat16_rn(-bs[i] * x[r]);
      }
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

    // ---- phase 6: W = bT K (bf16, rows 0..63 of WQ); S^T -> bf16 (bT V stays in TMEM)
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
        float ws[16], ut[16];
        tmem_ld16(tmem + lane_base + COL_DC + 16 * q, ws);
        tmem_ld16(tmem + lane_base + COL_D2 + 128 + 16 * q, ut);
        tmem_ld_wait();
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int o = 16 * q + 8 * half;
          const int u = 8 * half;
          uint4 pk;
          pk.x = pack_bf16(ut[u + 0] - ws[u + 0] * inv64, ut[u + 1] - ws[u + 1] * inv64);
          pk.y = pack_bf16(ut[u + 2] - ws[u + 2] * inv64, ut[u + 3] - ws[u + 3] * inv64);
          pk.z = pack_bf16(ut[u + 4] - ws[u + 4] * inv64, ut[u + 5] - ws[u + 5] * inv64);
          pk.w = pack_bf16(ut[u + 6] - ws[u + 6] * inv64, ut[u + 7] - ws[u + 7] * inv64);
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
