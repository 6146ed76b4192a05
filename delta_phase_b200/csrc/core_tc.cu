// Tensor-core (tcgen05) chunkwise complex delta-rule forward for d_k = d_v = 64,
// bf16 inputs, fp32 accumulation.
//
// Reference: _chunkwise_delta_reference (delta_phase/kernels/triton_chunk_delta.py:211-252)
// and the core of DeltaPhaseHolographicBlock.forward (delta_phase/layers.py:203-236).
//
// Real form (see core_simt.cu): per chunk of 64 tokens with key features K (64 x 128,
// interleaved cos/sin), query features Q, values V, write strengths beta and the state
// S (64 x 128, fp32, kept transposed in tensor memory for the whole sequence):
//   A = strict_lower(K K^T / 64) diag(beta),  bT = diag(beta) (I + A)^-1,  P = tril(Q K^T)
//   E = V - K S^T / 64;  U = bT E;  O = (Q S^T + P U) / 64;  S^T += K^T U
// (U = bT V - (bT K) S^T / 64 of the WY form, with the state correction applied before
// the triangular factor, so no bT [K | V] product is needed.)
//
// Two warp-specialised roles share one CTA per (batch, head):
//   * prep (8 warps) computes the state-independent work of chunk c+1 while
//   * chain (4 warps) runs the recurrence of chunk c.
// Prep: phasors (bf16) from TMA-loaded inputs; G1 = [K; Q] K^T (tcgen05, M=128); A and P
// from the Gram rows; T = (I + A)^-1 in fp32 (16 x 16 diagonal blocks by right-looking
// substitution, the 16 -> 32 block merge on warp-level tf32 MMA) into a per-slot buffer.
// Chain: S^T -> bf16; G3 = [K; Q] S^T (M=128) and, while it runs, the 32 -> 64 merge of
// the inverse; E and bT = diag(beta) T in bf16 (two warps each); U = bT E (M=64);
// G4 S^T += K^T U
// (M=128, accumulated in TMEM) and G5: Q S^T += P U (M=128 with A starting 64 rows before
// P, so the product lands in the Q rows of G3's accumulator); outputs.  Buffers the chain
// reads are double-buffered; hand-off uses mbarriers (ready / free per slot).
// Operand tiles use the SWIZZLE_NONE core-matrix layout (8 rows x 16 bytes), so one
// buffer is a K-major or MN-major operand by swapping the two descriptor strides: K is
// read as A and B of G1, A of G3 and A^T of G4 without copies.  M=64 accumulators put
// row m in TMEM lane (m % 16) + 32 (m / 16).  Every wait is bounded.
#include <cstring>

#include "dp_common.cuh"
#include "tc_ptx.cuh"
#include "tmap.cuh"

namespace dp {

int *device_error_ptr();

namespace {

using namespace ptx;

constexpr int kC = 64;     // tokens per chunk
constexpr int kF = 128;    // key features (2 * d_k)
constexpr int kDv = 64;    // value channels
constexpr int kPrepThreads = 256;   // warps 0..7
constexpr int kChainThreads = 128;  // warps 8..11
constexpr int kThreads = kPrepThreads + kChainThreads;
constexpr int BAR_PREP = 1, BAR_CHAIN = 2;
constexpr uint64_t kTimeoutNs = 2000000000ull;  // 2 s per wait

// shared-memory map (bytes).  bf16 tiles: row group (8 rows) of a 128- or 64-wide tile.
constexpr int RG_KQ = 16 * 128;
constexpr int RG_64 = 8 * 128;
constexpr int KQ_BYTES = 16 * RG_KQ;                 // rows 0..63 K, rows 64..127 Q
constexpr int BT_BYTES = 8 * RG_64;                  // bT = diag(beta) (I + A)^-1, bf16
constexpr int V_BYTES = 8 * RG_64;                   // V, then E = V - K S^T / 64 (chain)
constexpr int P_BYTES = 8 * RG_64;
constexpr int OFF_KQ = 0;                            // [2 slots]
constexpr int OFF_BT = OFF_KQ + 2 * KQ_BYTES;        // [2 slots]
constexpr int OFF_VS = OFF_BT + 2 * BT_BYTES;        // [2 slots]
constexpr int OFF_P = OFF_VS + 2 * V_BYTES;          // [2 slots]; 8 KB of shared memory precede it
constexpr int OFF_U = OFF_P + 2 * P_BYTES;           // chain only
constexpr int OFF_S0 = OFF_U + 8 * RG_64;            // S^T bf16 (128 x 64), chain only
constexpr int OFF_STAGE = OFF_S0 + 16 * RG_64;       // raw theta_k, theta_q, v rows of a chunk
constexpr int STAGE_BYTES = 3 * kC * 128;
constexpr int LDA = 68;                              // padded fp32 row stride
constexpr int OFF_AT = OFF_STAGE + STAGE_BYTES;      // A^T fp32: At[k][i] = A[i][k]
constexpr int TF_FLOATS = kC * LDA;
constexpr int OFF_TF = OFF_AT + kC * LDA * 4;        // T = (I + A)^-1 fp32, [2 slots] (chain forms bT)
constexpr int LDZ = 36;
constexpr int OFF_Z = OFF_TF + 2 * TF_FLOATS * 4;    // block-merge scratch fp32 (32 x LDZ)
constexpr int OFF_BETA = OFF_Z + 32 * LDZ * 4;       // beta, 2 chunk slots
constexpr int OFF_BSLOT = OFF_BETA + 2 * kC * 4;     // beta (complex beta: Re) of each slot's chunk (chain)
constexpr int OFF_BIM = OFF_BSLOT + 2 * kC * 4;      // complex beta: Im(beta) of each slot's chunk (chain)
constexpr int LDA10 = 36;
constexpr int A10_FLOATS = 32 * LDA10;
constexpr int OFF_A10 = OFF_BIM + 2 * kC * 4;         // A block (rows 32.., cols ..32) for the chain's merge [2]
constexpr int OFF_BAR = OFF_A10 + 2 * A10_FLOATS * 4;
constexpr int SMEM_BYTES = OFF_BAR + 128;
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
// complex beta: the write-key tile W (64 x 128 bf16, RG_KQ row groups) lives in the A^T
// buffer for the prep role's Gram MMA and in the S^T operand buffer for the chain's update
static_assert(KQ_BYTES / 2 <= kC * LDA * 4 && KQ_BYTES / 2 <= 16 * RG_64, "W tile fits its aliases");

// tensor-memory columns (fp32)
constexpr uint32_t COL_S = 0;      // S^T, M = 128 (lane = feature)
constexpr uint32_t COL_D1 = 64;    // [K;Q] K^T, M = 128 (prep)
constexpr uint32_t COL_R3 = 128;   // [K;Q] S^T, M = 128; rows 64.. then += P U (chain)
constexpr uint32_t COL_RU = 192;   // U = bT E, M = 64 (chain)
constexpr uint32_t TMEM_COLS = 256;

__device__ __forceinline__ uint32_t cm_off(int r, int k, int rg) {
  return (uint32_t)((r >> 3) * rg + (k >> 3) * 128 + (r & 7) * 16 + (k & 7) * 2);
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&h);
}

// Operand tiles: bf16 for the real-beta rule; fp16 (F16) for the complex-beta rule, whose
// update is isometric, so the per-chunk rounding of the tiles is not damped and adds up
// along the sequence like a random walk (bf16 tiles: 1.3e-2 relative L2 after 1000
// tokens; fp16 tiles: 1.6e-3).  fp16 operands are kept in range by scaling S and P by
// 1 / 64 (exact); values past 65504 set `over`, reported as DP_ERR_RANGE.
template <bool F16>
__device__ __forceinline__ uint32_t pack_op(float a, float b) {
  if (F16) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
  }
  return pack_bf16(a, b);
}
template <bool F16>
__device__ __forceinline__ uint32_t pack_chk(float a, float b, bool &over) {
  if (F16) over |= !(fabsf(a) <= 65504.f) || !(fabsf(b) <= 65504.f);
  return pack_op<F16>(a, b);
}
template <bool F16>
__device__ __forceinline__ float2 unpack_op(uint32_t w) {
  if (F16) return __half22float2(*reinterpret_cast<const __half2 *>(&w));
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w));
}
template <bool F16>
__host__ __device__ constexpr uint32_t idesc_op(int M, int N, bool a_mn_major, bool b_mn_major) {
  return F16 ? idesc_f16(M, N, a_mn_major, b_mn_major) : idesc_bf16(M, N, a_mn_major, b_mn_major);
}

// Complex beta: one (cos, sin) pair of a key phasor (fp16x2) times beta = br + i bi, i.e.
// the write key (br c - bi s, br s + bi c), rounded to fp16.  The prep and chain roles
// both form W through this function from the same key words, so they agree bit for bit.
__device__ __forceinline__ uint32_t rotate_pair(uint32_t cs, float br, float bi) {
  const float2 f = unpack_op<true>(cs);
  return pack_op<true>(fmaf(br, f.x, -bi * f.y), fmaf(br, f.y, bi * f.x));
}

// sin/cos of a phase: reduce to [-pi, pi] (x - 2 pi round(x / 2 pi), with the rounding
// done on the FMA pipe by the 1.5 * 2^23 trick and 2 pi split in two parts), then the
// hardware approximation; the error is far below bf16 resolution.
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

// Warp-level tf32 MMA (to_tf32, mma_tf32_m16n8k8: tc_ptx.cuh) for the small block products of
// the triangular inverse: operands straight from shared memory into registers, no tensor
// memory round trip.

// One warp: D[16 x 16] = X[16 x K] Y[K x 16], X(i, k) = x[i * xs_i + k * xs_k],
// Y(k, j) = y[k * ys_k + j * ys_j] (fp32 in shared memory, tf32 products); D is
// returned as two m16n8 fragments.
template <int K>
__device__ __forceinline__ void warp_gemm16(float (&d0)[4], float (&d1)[4], const float *x, int xs_i, int xs_k,
                                            const float *y, int ys_k, int ys_j, int lane) {
  const int g = lane >> 2, c = lane & 3;
#pragma unroll
  for (int i = 0; i < 4; ++i) d0[i] = d1[i] = 0.f;
#pragma unroll
  for (int k0 = 0; k0 < K; k0 += 8) {
    const uint32_t a[4] = {to_tf32(x[g * xs_i + (k0 + c) * xs_k]), to_tf32(x[(g + 8) * xs_i + (k0 + c) * xs_k]),
                           to_tf32(x[g * xs_i + (k0 + c + 4) * xs_k]),
                           to_tf32(x[(g + 8) * xs_i + (k0 + c + 4) * xs_k])};
    const uint32_t b0[2] = {to_tf32(y[(k0 + c) * ys_k + g * ys_j]), to_tf32(y[(k0 + c + 4) * ys_k + g * ys_j])};
    const uint32_t b1[2] = {to_tf32(y[(k0 + c) * ys_k + (g + 8) * ys_j]),
                            to_tf32(y[(k0 + c + 4) * ys_k + (g + 8) * ys_j])};
    mma_tf32_m16n8k8(d0, a, b0);
    mma_tf32_m16n8k8(d1, a, b1);
  }
}

// Stores a warp's 16 x 16 result (two m16n8 fragments) scaled by `sc` at out[i * ld + j].
__device__ __forceinline__ void warp_store16(float *out, int ld, const float (&d0)[4], const float (&d1)[4], float sc,
                                             int lane) {
  const int g = lane >> 2, c = lane & 3;
  *reinterpret_cast<float2 *>(out + g * ld + 2 * c) = make_float2(sc * d0[0], sc * d0[1]);
  *reinterpret_cast<float2 *>(out + (g + 8) * ld + 2 * c) = make_float2(sc * d0[2], sc * d0[3]);
  *reinterpret_cast<float2 *>(out + g * ld + 8 + 2 * c) = make_float2(sc * d1[0], sc * d1[1]);
  *reinterpret_cast<float2 *>(out + (g + 8) * ld + 8 + 2 * c) = make_float2(sc * d1[2], sc * d1[3]);
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
  int use_tmap;            // load chunks through the tensor maps below
  ChunkMapDims mdims[3];   // per input: the map dimension of token, head and batch
};

// Tensor maps of theta_k, theta_q, v (tmap.cuh): one chunk of one (b, h) per copy.
struct alignas(64) TcMaps {
  CUtensorMap m[3];
};

// Copies of chunk rows [c0, c0 + n) of one (b, h) into the stage (one full warp; lane 0
// registers the expected bytes first).  With tensor maps (L >= 64): one tiled copy per
// tensor (rows past L arrive as zeros and are not used) -- measured faster than both
// alternatives, for contiguous inputs and for the (B, L, H, d_k) projection views of a
// block; otherwise contiguous rows are one bulk copy per tensor, other layouts one bulk
// copy per row.
__device__ __forceinline__ void issue_chunk_loads(const TcArgs &a, const TcMaps &maps, int b, int h, int c0, int n,
                                                  uint8_t *stage, uint64_t *bar, int lane) {
  if (a.use_tmap) {
    if (lane == 0) {
      mbar_arrive_expect_tx(bar, (uint32_t)(3 * kC * 128));
#pragma unroll
      for (int x = 0; x < 3; ++x) tma_load_chunk(stage + x * kC * 128, &maps.m[x], a.mdims[x], c0, h, b, bar);
    }
    return;
  }
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

struct Bars {
  uint64_t load, prep_mma, chain_mma, ready[2], free_[2];
};

// ------------------------------------------------------------------------------ prep
// Returns false if a bounded wait expired (after letting its own copies / MMAs land).
// CB: complex beta (beta = 1 + e^{i phi}, a.beta holds phi): G1 = [K; Q] W^T with the
// write key W = beta K, A[i][k] = K_i . W_k / 64 (not symmetric; no beta factor left).
template <bool CB>
__device__ bool prep_role(const TcArgs &a, const TcMaps &maps, uint8_t *smem, Bars *bars, uint32_t tmem, int b, int h,
                          int nchunks) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q = warp & 3, hf = warp >> 2;  // TMEM lane quarter, column half
  const uint32_t lane_base = (uint32_t)(q * 32) << 16;
  const int L = a.L;
  uint8_t *stage = smem + OFF_STAGE;
  float *at = reinterpret_cast<float *>(smem + OFF_AT);
  float *tf0 = reinterpret_cast<float *>(smem + OFF_TF);
  float *zs = reinterpret_cast<float *>(smem + OFF_Z);
  float *bs2 = reinterpret_cast<float *>(smem + OFF_BETA);
  const float inv64 = 1.0f / 64.0f;

  int issued = 0, consumed = 0;
  uint32_t pm_phase = 0;
  bool mma_pending = false, ok = true;
  if (nchunks > 0) {
    if (warp == 0) issue_chunk_loads(a, maps, b, h, 0, min(kC, L), stage, &bars->load, lane);
    issued = 1;
  }
  if (tid < kC)
    bs2[tid] = (tid < L) ? load_beta(a.beta, a.beta_dt, b * a.s_b.b + h * a.s_b.h + (int64_t)tid * a.s_b.t) : 0.f;
  group_sync(BAR_PREP, kPrepThreads);

  for (int c = 0; c < nchunks; ++c) {
    const int slot = c & 1, t0 = c * kC, nvalid = min(kC, L - t0);
    uint8_t *kq = smem + OFF_KQ + slot * KQ_BYTES;
    uint8_t *vb = smem + OFF_VS + slot * V_BYTES;
    float *tf = tf0 + slot * TF_FLOATS;
    uint8_t *pb = smem + OFF_P + slot * P_BYTES;
    const float *bs = bs2 + slot * kC;

    // the chain must be done with this slot (chunk c - 2)
    // one thread polls the mbarriers; the others wait in the hardware barrier
    if (tid == 0) {
      if (c >= 2) ok = mbar_wait(&bars->free_[slot], (uint32_t)(((c - 2) >> 1) & 1), kTimeoutNs);
      if (ok) ok = mbar_wait(&bars->load, (uint32_t)(c & 1), kTimeoutNs);
    }
    if (group_any(!ok, BAR_PREP, kPrepThreads)) { ok = false; break; }
    consumed = c + 1;

    // ---- P1: phasors (bf16) -> K, Q tiles; values -> V tile; beta of the next chunk.
    //      Warp w covers token rows 8w .. 8w+7, lane l = 8a + b: row 8w + b, channel
    //      segment (a + 2b + 4r) % 8 in pass r.  Each load from the staged rows then hits
    //      every 16-byte bank group 4 times (segment), and so does each store into the
    //      core-matrix tiles (row % 8): both are conflict-free 512-byte accesses.
    {
      uint32_t bnext = 0u;  // raw bits; converted at the store below, after the phasor work
      if (tid < kC && t0 + kC + tid < L)
        bnext = load_raw_scalar(a.beta, a.beta_dt, b * a.s_b.b + h * a.s_b.h + (int64_t)(t0 + kC + tid) * a.s_b.t);
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int t = 8 * warp + (lane & 7), sg = ((lane >> 3) + 2 * (lane & 7) + 4 * r) & 7;
        const bool valid = t < nvalid;
        float br = 1.f, bi = 0.f;
        if (CB) {
          fast_sincos(bs[t], &bi, &br);
          br += 1.f;
        }
        uint4 kraw = make_uint4(0, 0, 0, 0), qraw = kraw, vraw = kraw;
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
          kw[2 * i] = pack_op<CB>(c0_, s0_);
          kw[2 * i + 1] = pack_op<CB>(c1_, s1_);
          const __nv_bfloat162 qq2 = *reinterpret_cast<const __nv_bfloat162 *>(&qr[i]);
          fast_sincos(__low2float(qq2), &s0_, &c0_);
          fast_sincos(__high2float(qq2), &s1_, &c1_);
          qw[2 * i] = pack_op<CB>(c0_, s0_);
          qw[2 * i + 1] = pack_op<CB>(c1_, s1_);
        }
        if (!valid) {
#pragma unroll
          for (int i = 0; i < 8; ++i) kw[i] = qw[i] = 0u;
        }
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          *reinterpret_cast<uint4 *>(kq + cm_off(t, 16 * sg + 8 * half, RG_KQ)) =
              make_uint4(kw[4 * half], kw[4 * half + 1], kw[4 * half + 2], kw[4 * half + 3]);
          *reinterpret_cast<uint4 *>(kq + cm_off(64 + t, 16 * sg + 8 * half, RG_KQ)) =
              make_uint4(qw[4 * half], qw[4 * half + 1], qw[4 * half + 2], qw[4 * half + 3]);
          if (CB)  // write key W = beta K into the (free) A^T buffer, for G1
            *reinterpret_cast<uint4 *>(smem + OFF_AT + cm_off(t, 16 * sg + 8 * half, RG_KQ)) =
                make_uint4(rotate_pair(kw[4 * half], br, bi), rotate_pair(kw[4 * half + 1], br, bi),
                           rotate_pair(kw[4 * half + 2], br, bi), rotate_pair(kw[4 * half + 3], br, bi));
        }
        *reinterpret_cast<uint4 *>(vb + cm_off(t, 8 * sg, RG_64)) = vraw;
      }
      if (tid < kC) bs2[(slot ^ 1) * kC + tid] = raw_scalar_to_f32(bnext, a.beta_dt);
    }
    fence_proxy_async_smem();
    group_sync(BAR_PREP, kPrepThreads);

    // ---- P2: the stage is free -> next chunk's loads; G1 = [K; Q] K^T  (M=128, N=64)
    if (c + 1 < nchunks) {
      if (warp == 0) issue_chunk_loads(a, maps, b, h, t0 + kC, min(kC, L - t0 - kC), stage, &bars->load, lane);
      issued = c + 2;
    }
    if (tid == 0) {
      tc_fence_after();
      const uint32_t sa = smem_u32(kq), sb = CB ? smem_u32(smem + OFF_AT) : sa;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        mma_f16_ss(tmem + COL_D1, make_desc(sa + kk * 256, 128, RG_KQ), make_desc(sb + kk * 256, 128, RG_KQ),
                   idesc_op<CB>(128, 64, false, false), kk > 0);
      mma_commit(&bars->prep_mma);
    }
    mma_pending = true;
    if (tid == 0) ok = mbar_wait(&bars->prep_mma, pm_phase, kTimeoutNs);
    if (group_any(!ok, BAR_PREP, kPrepThreads)) { ok = false; break; }
    pm_phase ^= 1;
    mma_pending = false;
    tc_fence_after();

    // ---- P3: A^T from the (exactly symmetric) Gram rows, At[k][i] = beta_k G[k][i] / 64
    //      for i > k (quarters 0, 1); P = tril(Q K^T) in bf16 (quarters 2, 3).
    //      Warp half hf takes columns 32 hf .. 32 hf + 31.
    if (CB && q < 2) {
      // row i of K W^T: A[i][k] = G1[i][k] / 64 for k < i, stored as column i of A^T
      const int i = q * 32 + lane;
      float g[32];
      tmem_ld32_sync(tmem + lane_base + COL_D1 + 32 * hf, g);
#pragma unroll
      for (int kk = 0; kk < 32; ++kk) at[(32 * hf + kk) * LDA + i] = (32 * hf + kk < i) ? g[kk] * inv64 : 0.f;
    } else if (q < 2) {
      const int k = q * 32 + lane;
      const float bk = bs[k] * inv64;
      float g[32];
      tmem_ld32_sync(tmem + lane_base + COL_D1 + 32 * hf, g);
#pragma unroll
      for (int i = 0; i < 32; i += 4) {
        const int c0 = 32 * hf;
        float4 w;
        w.x = (c0 + i + 0 > k) ? g[i + 0] * bk : 0.f;
        w.y = (c0 + i + 1 > k) ? g[i + 1] * bk : 0.f;
        w.z = (c0 + i + 2 > k) ? g[i + 2] * bk : 0.f;
        w.w = (c0 + i + 3 > k) ? g[i + 3] * bk : 0.f;
        *reinterpret_cast<float4 *>(at + k * LDA + c0 + i) = w;
      }
    } else {
      const int t = (q - 2) * 32 + lane;
      float p[32];
      tmem_ld32_sync(tmem + lane_base + COL_D1 + 32 * hf, p);
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int c0 = 32 * hf + 16 * u;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int s = c0 + 8 * half;
          const float *pp = p + 16 * u + 8 * half;
          const float ps = CB ? inv64 : 1.f;  // fp16 tiles hold P / 64
          uint4 w;
          w.x = pack_op<CB>(s + 0 <= t ? pp[0] * ps : 0.f, s + 1 <= t ? pp[1] * ps : 0.f);
          w.y = pack_op<CB>(s + 2 <= t ? pp[2] * ps : 0.f, s + 3 <= t ? pp[3] * ps : 0.f);
          w.z = pack_op<CB>(s + 4 <= t ? pp[4] * ps : 0.f, s + 5 <= t ? pp[5] * ps : 0.f);
          w.w = pack_op<CB>(s + 6 <= t ? pp[6] * ps : 0.f, s + 7 <= t ? pp[7] * ps : 0.f);
          *reinterpret_cast<uint4 *>(pb + cm_off(t, s, RG_64)) = w;
        }
      }
      fence_proxy_async_smem();  // P is an MMA operand of the chain (G5)
    }
    tc_fence_before();
    group_sync(BAR_PREP, kPrepThreads);

    // ---- P4a: 16 x 16 diagonal blocks of (I + A)^-1, right-looking substitution with
    //      the column in registers (threads 0..63: block tid / 16, column tid % 16)
    if (tid >= 64) {
      // beside the diagonal solves: the block of A^T the chain's 32 -> 64 merge reads,
      // a10[k][i] = At[k][32 + i] (k, i < 32), to this slot's buffer
      float *a10 = reinterpret_cast<float *>(smem + OFF_A10) + slot * A10_FLOATS;
      for (int e = tid - 64; e < 32 * 8; e += kPrepThreads - 64) {
        const int k = e >> 3, i4 = 4 * (e & 7);
        *reinterpret_cast<float4 *>(a10 + k * LDA10 + i4) = *reinterpret_cast<const float4 *>(at + k * LDA + 32 + i4);
      }
    }
    if (tid < 64) {
      const int o = 16 * (tid >> 4), col = tid & 15;
      float cl[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) cl[i] = (i == col) ? 1.f : 0.f;
#pragma unroll
      for (int k = 0; k < 15; ++k) {
        const float tk = cl[k];
        const float *ak = at + (o + k) * LDA + o;
#pragma unroll
        for (int i4 = ((k + 1) & ~3); i4 < 16; i4 += 4) {
          const float4 av = *reinterpret_cast<const float4 *>(ak + i4);
          if (i4 + 0 > k) cl[i4 + 0] = fmaf(-av.x, tk, cl[i4 + 0]);
          if (i4 + 1 > k) cl[i4 + 1] = fmaf(-av.y, tk, cl[i4 + 1]);
          if (i4 + 2 > k) cl[i4 + 2] = fmaf(-av.z, tk, cl[i4 + 2]);
          if (i4 + 3 > k) cl[i4 + 3] = fmaf(-av.w, tk, cl[i4 + 3]);
        }
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) tf[(o + i) * LDA + o + col] = cl[i];
    }
    group_sync(BAR_PREP, kPrepThreads);

    // ---- P4b: 16 -> 32 merge for the block pairs (0,1), (2,3) on warps 0, 1 (tf32 mma):
    //      Z = A[16+i][k] T[k][j], then T[16+i][j] = -T11 Z
    if (warp < 2) {
      const int o = 32 * warp;
      float d0[4], d1[4];
      warp_gemm16<16>(d0, d1, at + o * LDA + o + 16, 1, LDA, tf + o * LDA + o, LDA, 1, lane);
      warp_store16(zs + 16 * warp * LDZ, LDZ, d0, d1, 1.f, lane);
      __syncwarp();
      warp_gemm16<16>(d0, d1, tf + (o + 16) * LDA + o + 16, LDA, 1, zs + 16 * warp * LDZ, LDZ, 1, lane);
      warp_store16(tf + (o + 16) * LDA + o, LDA, d0, d1, -1.f, lane);
    }
    group_sync(BAR_PREP, kPrepThreads);

    // ---- P4d: beta of this chunk next to T for the chain, which forms bT = diag(beta) T
    if (tid < kC) {
      if (CB) {
        float sp, cp;
        fast_sincos(bs[tid], &sp, &cp);
        reinterpret_cast<float *>(smem + OFF_BSLOT)[slot * kC + tid] = 1.f + cp;
        reinterpret_cast<float *>(smem + OFF_BIM)[slot * kC + tid] = sp;
      } else {
        reinterpret_cast<float *>(smem + OFF_BSLOT)[slot * kC + tid] = bs[tid];
      }
    }
    // T, beta, P, V and K, Q of this slot are ready for the chain (the tiles that MMAs read
    // were fenced for the async proxy where they were written)
    tc_fence_before();
    group_sync(BAR_PREP, kPrepThreads);
    if (tid == 0) mbar_arrive(&bars->ready[slot]);
  }

  if (!ok) {
    // let this role's own copies and MMAs land before shared / tensor memory is released
    if (tid == 0) {
      for (int k = consumed; k < issued; ++k) mbar_wait(&bars->load, (uint32_t)(k & 1), kTimeoutNs);
      if (mma_pending) mbar_wait(&bars->prep_mma, pm_phase, kTimeoutNs);
    }
  }
  return ok;
}

// ------------------------------------------------------------------------------ chain
// CB: complex beta; U = T E (no beta factor) and the state update S^T += W^T U, with W
// rebuilt from this slot's K tile into the S^T operand buffer while U = T E runs.
template <bool CB>
__device__ bool chain_role(const TcArgs &a, uint8_t *smem, Bars *bars, uint32_t tmem, int bh, int b,
                           int h, int nchunks) {
  const int ctid = threadIdx.x - kPrepThreads, cw = ctid >> 5, lane = ctid & 31;
  const uint32_t lane_base = (uint32_t)(cw * 32) << 16;
  const int L = a.L;
  uint8_t *ub = smem + OFF_U;
  uint8_t *s0 = smem + OFF_S0;
  const float inv64 = 1.0f / 64.0f;
  const int j = cw * 32 + lane;  // feature row of S^T held by this thread
  const int64_t sbase = (int64_t)bh * kDv * kF;

  // initial state^T -> TMEM
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    float vals[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) vals[i] = a.state_in ? a.state_in[sbase + (int64_t)(16 * u + i) * kF + j] : 0.f;
    tmem_st16(tmem + lane_base + COL_S + 16 * u, vals);
  }
  tmem_st_wait();
  tc_fence_before();
  group_sync(BAR_CHAIN, kChainThreads);

  uint32_t cm_phase = 0;
  bool ok = true, mma_pending = false, over = false;
  const float ss64 = CB ? inv64 : 1.f;  // fp16 tiles hold S^T / 64
  for (int c = 0; c < nchunks; ++c) {
    const int slot = c & 1, t0 = c * kC, nvalid = min(kC, L - t0);
    uint8_t *kq = smem + OFF_KQ + slot * KQ_BYTES;
    uint8_t *tb = smem + OFF_BT + slot * BT_BYTES;
    uint8_t *vs = smem + OFF_VS + slot * V_BYTES;
    uint8_t *pb = smem + OFF_P + slot * P_BYTES;
    float *tfs = reinterpret_cast<float *>(smem + OFF_TF) + slot * TF_FLOATS;
    const float *a10 = reinterpret_cast<const float *>(smem + OFF_A10) + slot * A10_FLOATS;
    const float *bsl = reinterpret_cast<const float *>(smem + OFF_BSLOT) + slot * kC;

    if (ctid == 0) ok = mbar_wait(&bars->ready[slot], (uint32_t)((c >> 1) & 1), kTimeoutNs);
    if (group_any(!ok, BAR_CHAIN, kChainThreads)) { ok = false; break; }
    tc_fence_after();

    // ---- C1: S^T (fp32, TMEM) -> bf16 operand tile
    {
      float sv[64];
      tmem_ld64_sync(tmem + lane_base + COL_S, sv);
#pragma unroll
      for (int u8 = 0; u8 < 8; ++u8) {
        const float *ss = sv + 8 * u8;
        *reinterpret_cast<uint4 *>(s0 + cm_off(j, 8 * u8, RG_64)) =
            make_uint4(pack_chk<CB>(ss[0] * ss64, ss[1] * ss64, over), pack_chk<CB>(ss[2] * ss64, ss[3] * ss64, over),
                       pack_chk<CB>(ss[4] * ss64, ss[5] * ss64, over), pack_chk<CB>(ss[6] * ss64, ss[7] * ss64, over));
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    group_sync(BAR_CHAIN, kChainThreads);

    // ---- C2: G3 = [K;Q] S^T -> R3  (M=128, N=64, K=128): rows 0..63 K S^T, 64.. Q S^T
    if (ctid == 0) {
      tc_fence_after();
      const uint32_t sa = smem_u32(kq), ss = smem_u32(s0);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        mma_f16_ss(tmem + COL_R3, make_desc(sa + kk * 256, 128, RG_KQ), make_desc(ss + kk * 2 * RG_64, RG_64, 128),
                   idesc_op<CB>(128, 64, false, true), kk > 0);
      mma_commit(&bars->chain_mma);
    }
    mma_pending = true;
    // ---- C2m: while G3 runs, the last level of the inverse: T[32+i][j] = -T11 (A10 T00)
    //      (tf32 mma, one 16 x 16 tile per warp; the U tile is the scratch)
    {
      float *zc = reinterpret_cast<float *>(ub);
      const int mi = 16 * (cw >> 1), nj = 16 * (cw & 1);
      float d0[4], d1[4];
      warp_gemm16<32>(d0, d1, a10 + mi, 1, LDA10, tfs + nj, LDA, 1, lane);
      warp_store16(zc + mi * LDZ + nj, LDZ, d0, d1, 1.f, lane);
      group_sync(BAR_CHAIN, kChainThreads);
      warp_gemm16<32>(d0, d1, tfs + (32 + mi) * LDA + 32, LDA, 1, zc + nj, LDZ, 1, lane);
      warp_store16(tfs + (32 + mi) * LDA + nj, LDA, d0, d1, -1.f, lane);
    }
    if (ctid == 0) ok = mbar_wait(&bars->chain_mma, cm_phase, kTimeoutNs);
    if (group_any(!ok, BAR_CHAIN, kChainThreads)) { ok = false; break; }
    cm_phase ^= 1;
    mma_pending = false;
    tc_fence_after();

    // ---- C3: E = V - K S^T / 64 -> bf16 in place of V (row t = lane of chain warps 0, 1).
    //      U = bT (V - K S^T / 64) = bT V - (bT K) S^T / 64: the state correction is applied
    //      before the triangular factor, so the prep role needs no bT [K | V] product.
    if (cw < 2) {
      const int t = 32 * cw + lane;
      float ks[64];
      tmem_ld64_sync(tmem + lane_base + COL_R3, ks);
#pragma unroll
      for (int u8 = 0; u8 < 8; ++u8) {
        uint4 *vp = reinterpret_cast<uint4 *>(vs + cm_off(t, 8 * u8, RG_64));
        const uint4 vr = *vp;
        const uint32_t vw[4] = {vr.x, vr.y, vr.z, vr.w};
        uint32_t ew[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 vv = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&vw[i]));
          if (CB)  // the state-read rows already carry the 1 / 64
            ew[i] = pack_chk<true>(vv.x - ks[8 * u8 + 2 * i], vv.y - ks[8 * u8 + 2 * i + 1], over);
          else
            ew[i] = pack_bf16(vv.x - ks[8 * u8 + 2 * i] * inv64, vv.y - ks[8 * u8 + 2 * i + 1] * inv64);
        }
        *vp = make_uint4(ew[0], ew[1], ew[2], ew[3]);
      }
    } else {
      // bT = diag(beta) T -> bf16 (row i = lane of chain warps 2, 3), beside E
      const int i = 32 * (cw - 2) + lane;
      const float bi = CB ? 1.f : bsl[i];
      const float *tr = tfs + i * LDA;
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8) {
        const float4 x0 = *reinterpret_cast<const float4 *>(tr + 8 * c8);
        const float4 x1 = *reinterpret_cast<const float4 *>(tr + 8 * c8 + 4);
        *reinterpret_cast<uint4 *>(tb + cm_off(i, 8 * c8, RG_64)) =
            make_uint4(pack_chk<CB>(bi * x0.x, bi * x0.y, over), pack_chk<CB>(bi * x0.z, bi * x0.w, over),
                       pack_chk<CB>(bi * x1.x, bi * x1.y, over), pack_chk<CB>(bi * x1.z, bi * x1.w, over));
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    group_sync(BAR_CHAIN, kChainThreads);

    // ---- C3u: U = bT E  (M=64, N=64, K=64) -> RU
    if (ctid == 0) {
      tc_fence_after();
      const uint32_t sb = smem_u32(tb), se = smem_u32(vs);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        mma_f16_ss(tmem + COL_RU, make_desc(sb + kk * 256, 128, RG_64), make_desc(se + kk * 2 * RG_64, RG_64, 128),
                   idesc_op<CB>(64, 64, false, true), kk > 0);
      mma_commit(&bars->chain_mma);
    }
    mma_pending = true;
    if (CB) {
      // W = beta K of this slot -> the S^T operand buffer (G3, its last reader, is done)
      const int t = ctid & 63;
      const float br = bsl[t], bi = reinterpret_cast<const float *>(smem + OFF_BIM)[slot * kC + t];
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        const uint32_t off = cm_off(t, 8 * (2 * jj + (ctid >> 6)), RG_KQ);
        const uint4 kr = *reinterpret_cast<const uint4 *>(kq + off);
        *reinterpret_cast<uint4 *>(s0 + off) = make_uint4(rotate_pair(kr.x, br, bi), rotate_pair(kr.y, br, bi),
                                                          rotate_pair(kr.z, br, bi), rotate_pair(kr.w, br, bi));
      }
    }
    if (ctid == 0) ok = mbar_wait(&bars->chain_mma, cm_phase, kTimeoutNs);
    if (group_any(!ok, BAR_CHAIN, kChainThreads)) { ok = false; break; }
    cm_phase ^= 1;
    mma_pending = false;
    tc_fence_after();

    // ---- C3c: U -> bf16 operand tile (M=64 rows: lanes < 16 of each quarter)
    {
      const int t = 16 * cw + lane;
      float uv[64];
      tmem_ld64_sync(tmem + lane_base + COL_RU, uv);
      if (lane < 16) {
#pragma unroll
        for (int u8 = 0; u8 < 8; ++u8) {
          const float *uu = uv + 8 * u8;
          *reinterpret_cast<uint4 *>(ub + cm_off(t, 8 * u8, RG_64)) =
              make_uint4(pack_chk<CB>(uu[0], uu[1], over), pack_chk<CB>(uu[2], uu[3], over),
                         pack_chk<CB>(uu[4], uu[5], over), pack_chk<CB>(uu[6], uu[7], over));
        }
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    group_sync(BAR_CHAIN, kChainThreads);

    // ---- C4: G4 S^T += K^T U (M=128) and G5 R3 += [X; P] U (M=128, A starting 8 KB
    //      before P: rows 64.. of R3 (Q S^T) gain P U; rows 0.. (K S^T, already used) are
    //      don't-care)
    if (ctid == 0) {
      tc_fence_after();
      const uint32_t sk = CB ? smem_u32(s0) : smem_u32(kq), su = smem_u32(ub), sp = smem_u32(pb) - 8 * RG_64;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint64_t ud = make_desc(su + kk * 2 * RG_64, RG_64, 128);
        mma_f16_ss(tmem + COL_S, make_desc(sk + kk * 2 * RG_KQ, RG_KQ, 128), ud, idesc_op<CB>(128, 64, true, true), 1u);
        mma_f16_ss(tmem + COL_R3, make_desc(sp + kk * 256, 128, RG_64), ud, idesc_op<CB>(128, 64, false, true), 1u);
      }
      mma_commit(&bars->chain_mma);
    }
    mma_pending = true;
    if (ctid == 0) ok = mbar_wait(&bars->chain_mma, cm_phase, kTimeoutNs);
    if (group_any(!ok, BAR_CHAIN, kChainThreads)) { ok = false; break; }
    cm_phase ^= 1;
    mma_pending = false;
    tc_fence_after();
    if (ctid == 0) mbar_arrive(&bars->free_[slot]);  // K, Q, T, beta, E, P of this slot are consumed

    // ---- C5: outputs O = R3 rows 64.. / 64 (row t = lane of chain warps 2, 3); the fp16
    //      tiles (S^T / 64, P / 64) put the 1 / 64 into R3 already
    if (cw >= 2) {
      const float ss64_out = CB ? 1.f : inv64;
      const int t = 32 * (cw - 2) + lane;
      float *orow = a.out + b * a.s_out.b + h * a.s_out.h + (int64_t)(t0 + t) * a.s_out.t;
      float o[64];
      tmem_ld64_sync(tmem + lane_base + COL_R3, o);
      if (t < nvalid) {
#pragma unroll
        for (int i = 0; i < 64; i += 4)
          *reinterpret_cast<float4 *>(orow + i) =
              make_float4(o[i] * ss64_out, o[i + 1] * ss64_out, o[i + 2] * ss64_out, o[i + 3] * ss64_out);
      }
    }
    tc_fence_before();
  }

  if (ok) {
    // final state: TMEM S^T -> complex64 state (row o, interleaved column j)
    tc_fence_after();
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float sv[16];
      tmem_ld16(tmem + lane_base + COL_S + 16 * u, sv);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 16; ++i) a.state_out[sbase + (int64_t)(16 * u + i) * kF + j] = sv[i];
    }
  } else if (mma_pending && ctid == 0) {
    mbar_wait(&bars->chain_mma, cm_phase, kTimeoutNs);
  }
  if (CB && over) atomicCAS(a.err, 0, DP_ERR_RANGE);
  return ok;
}

template <bool CB>
__global__ void __launch_bounds__(kThreads, 1) core_tc_kernel(const __grid_constant__ TcArgs a,
                                                               const __grid_constant__ TcMaps maps) {
  extern __shared__ __align__(1024) uint8_t smem[];
  Bars *bars = reinterpret_cast<Bars *>(smem + OFF_BAR);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 1);
  int *fail_flag = reinterpret_cast<int *>(tmem_slot + 1);
  float *tf = reinterpret_cast<float *>(smem + OFF_TF);

  const int tid = threadIdx.x, warp = tid >> 5;
  const int bh = blockIdx.x, b = bh / a.H, h = bh % a.H;
  const int nchunks = (a.L + kC - 1) / kC;

  if (tid == 0) {
    mbar_init(&bars->load, 1);
    mbar_init(&bars->prep_mma, 1);
    mbar_init(&bars->chain_mma, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->ready[i], 1);
      mbar_init(&bars->free_[i], 1);
    }
    *fail_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  // T's strictly upper blocks are never written: zero them once (both slots)
  for (int i = tid; i < 2 * TF_FLOATS; i += kThreads) tf[i] = 0.f;
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  bool ok;
  if (tid < kPrepThreads)
    ok = prep_role<CB>(a, maps, smem, bars, tmem, b, h, nchunks);
  else
    ok = chain_role<CB>(a, smem, bars, tmem, bh, b, h, nchunks);
  if (!ok) atomicExch(fail_flag, 1);

  tc_fence_before();
  __syncthreads();
  if (tid == 0 && *fail_flag) atomicCAS(a.err, 0, DP_ERR_TIMEOUT);
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

bool core_fwd_pipe(const void *tk, const void *tq, const void *v, const void *beta, int beta_dt,
                   const float *state_in, float *out, float *state_out, int B, int H, int L, const SeqStrides *s,
                   cudaStream_t stream, bool cbeta, int *rc);

// cbeta: `beta` holds phi of the complex beta 1 + e^{i phi} (ComplexBetaDeltaPhaseBlock).
// L >= 64 runs the pipelined kernel of core_pipe.cu (both modes); the kernel below takes
// shorter sequences.
int core_fwd_tc(const void *tk, const void *tq, const void *v, const void *beta, int beta_dt,
                const float *state_in, float *out, float *state_out, int B, int H, int L,
                const SeqStrides *s, cudaStream_t stream, bool cbeta) {
  {
    int rc = DP_OK;
    if (core_fwd_pipe(tk, tq, v, beta, beta_dt, state_in, out, state_out, B, H, L, s, stream, cbeta, &rc)) return rc;
  }
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
  TcMaps maps;
  memset(&maps, 0, sizeof(maps));
  const void *base[3] = {tk, tq, v};
  a.use_tmap = L >= kC;
  for (int x = 0; x < 3 && a.use_tmap; ++x)
    a.use_tmap = encode_chunk_map(&maps.m[x], &a.mdims[x], base[x], B, H, L, s[x]);
  auto kern = cbeta ? core_tc_kernel<true> : core_tc_kernel<false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  if (e != cudaSuccess) return set_error(DP_ERR_CUDA, std::string("core_tc smem attr: ") + cudaGetErrorString(e));
  kern<<<B * H, kThreads, SMEM_BYTES, stream>>>(a, maps);
  return check_launch("core_tc_kernel");
}

}  // namespace dp
