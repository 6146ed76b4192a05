// Pipelined tensor-core (tcgen05) chunkwise complex delta-rule forward for d_k = d_v = 64,
// bf16 inputs, real beta, fp32 accumulation.
//
// Reference: _chunkwise_delta_reference (delta_phase/kernels/triton_chunk_delta.py:211-252)
// and the core of DeltaPhaseHolographicBlock.forward (delta_phase/layers.py:203-236).
//
// Per 64-token chunk, in the real form of core_simt.cu (K, Q: 64 x 128 interleaved cos/sin
// features, S the 64 x 128 fp32 state, kept transposed in tensor memory):
//   A = strict_lower(K K^T / 64) diag(beta),  bT = diag(beta) (I + A)^-1,  P = tril(Q K^T)
//   E = V - K S^T / 64;  U = bT E;  O = (Q S^T + P U) / 64;  S^T += K^T U
//
// The work of a chunk is split over three warp-specialised roles that run three chunks at
// once, so the per-chunk latencies of the roles overlap instead of adding up:
//   * phasor role (warps 0-7), chunk c + 2: two threads per row of [K; Q] compute its 64
//     phasors from the TMA-loaded phases (two stages: the next chunk's phases are in flight)
//     and store the row straight into tensor memory (the A operand of G1 and G3: no
//     shared-memory traffic for Q at all), the K rows also into a shared-memory tile (B of
//     G1, A^T of G4); then G1 = [K; Q] K^T (tcgen05, M = 128, A from tensor memory).  Its
//     warps of TMEM lane quarters 2 and 3 also store the outputs of chunk c - 1 (read out of
//     tensor memory into a swizzled tile, then two bulk tensor stores) and free the chain's
//     accumulator slot;
//   * inverse role (warps 8-11), chunk c + 1: A and P from the G1 rows, T = (I + A)^-1 in
//     fp32 (16 x 16 diagonal blocks by forward substitution with the next row prefetched,
//     the 16 -> 32 and 32 -> 64 block merges on warp-level tf32 MMA), bT in bf16;
//   * chain role (warps 12-19), chunk c: the state recurrence.  S^T -> bf16; G3 = [K; Q] S^T
//     (M = 128, A from tensor memory); E; U = bT E (M = 64); G4: S^T += K^T U, waited for on
//     its own, and G5: Q S^T += P U (M = 128, A starting 64 rows before P) behind it.  A
//     second thread of the role issues the V loads (TMA straight into the operand tile,
//     eight 16-byte column groups per chunk, two chunks ahead) and waits for the next
//     chunk's inputs while thread 0 waits for this chunk's MMAs.
// Every MMA is issued by one lane that elect.sync picks in warp-uniform code (a plain lane-0
// branch measured about twice as slow per MMA).  Hand-offs between roles are mbarriers only
// (the chain's MMA commits arrive on the barriers that free the phasor and inverse roles'
// slots); K and Q live in a ring of three slots (written two chunks ahead of the chain),
// the inverse role's outputs, V and the G3 accumulator in rings of two.  Every wait is
// bounded: on expiry the kernel records DP_ERR_TIMEOUT, lets its own copies and MMAs land
// and frees its tensor memory.
#include <cstring>

#include "dp_common.cuh"
#include "tc_ptx.cuh"
#include "tmap.cuh"

namespace dp {

int *device_error_ptr();

namespace {

using namespace ptx;

constexpr int kC = 64;   // tokens per chunk
constexpr int kF = 128;  // key features (2 * d_k)
constexpr int kDv = 64;  // value channels
constexpr int kPhThreads = 256;   // warps 0-7
constexpr int kInvThreads = 128;  // warps 8-11
constexpr int kChThreads = 256;   // warps 12-19
constexpr int kInvBase = kPhThreads, kChBase = kPhThreads + kInvThreads;
constexpr int kThreads = kChBase + kChThreads;
constexpr int BAR_PH = 1, BAR_INV = 2, BAR_CH = 3, BAR_OUT = 4;
constexpr int NKQ = 3;                           // K / Q tile ring
constexpr uint64_t kTimeoutNs = 2000000000ull;   // 2 s per wait

// shared-memory map (bytes).  bf16 tiles in the SWIZZLE_NONE core-matrix layout: a row
// group (8 rows) of a 128-wide tile is RG_KQ bytes, of a 64-wide tile RG_64.
constexpr int RG_KQ = 16 * 128;
constexpr int RG_64 = 8 * 128;
constexpr int K_BYTES = 8 * RG_KQ;                   // K tile: 64 rows x 128 features
constexpr int T64_BYTES = 8 * RG_64;                 // one 64 x 64 bf16 tile
constexpr int OFF_K = 0;                             // [NKQ]
constexpr int OFF_STAGE = OFF_K + NKQ * K_BYTES;     // [2] theta_k rows 0..63, theta_q rows 64..127 (128-byte swizzle)
constexpr int STAGE_BYTES = 2 * kC * 128;
static_assert(OFF_STAGE % 1024 == 0 && STAGE_BYTES % 1024 == 0, "the swizzled stages must be 1024-byte aligned");
constexpr int OFF_V = OFF_STAGE + 2 * STAGE_BYTES;   // [2] V, then E (column-group-major layout)
constexpr int OFF_BT = OFF_V + 2 * T64_BYTES;        // [2] bT = diag(beta) T, bf16
constexpr int OFF_P = OFF_BT + 2 * T64_BYTES;        // [2] P; 8 KB of shared memory precede each slot
constexpr int OFF_U = OFF_P + 2 * T64_BYTES;         // chain: U bf16
constexpr int OFF_S0 = OFF_U + T64_BYTES;            // chain: S^T bf16 (128 x 64)
constexpr int OFF_OUT = OFF_S0 + 16 * RG_64;         // chain: outputs of a chunk, two 64 x 32 fp32 boxes (128-byte swizzle)
constexpr int OUT_BYTES = 2 * kC * 128;
static_assert(OFF_OUT % 1024 == 0, "the swizzled output tile must be 1024-byte aligned");
constexpr int LDA = 68;                              // padded fp32 row stride
constexpr int OFF_AT = OFF_OUT + OUT_BYTES;          // inverse role: A^T fp32, At[k][i] = A[i][k]
constexpr int OFF_TF = OFF_AT + kC * LDA * 4;        // inverse role: T = (I + A)^-1 fp32
constexpr int LDZ = 36;
constexpr int OFF_Z = OFF_TF + kC * LDA * 4;         // inverse role: block-merge scratch (32 x LDZ)
constexpr int OFF_BETA = OFF_Z + 32 * LDZ * 4;       // inverse role: beta of its chunk
constexpr int OFF_BAR = OFF_BETA + kC * 4;
constexpr int SMEM_BYTES = OFF_BAR + 256;
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
static_assert(OFF_P == OFF_BT + 2 * T64_BYTES, "G5 reads the 8 KB before a P slot as don't-care rows");

// tensor-memory columns (32-bit)
constexpr uint32_t COL_S = 0;      // S^T fp32, M = 128 (lane = feature)
constexpr uint32_t COL_R3 = 64;    // [2] at 64, 128: [K;Q] S^T, then rows 64.. += P U (chain)
constexpr uint32_t COL_RU = 192;   // U = bT E, M = 64 (chain)
constexpr uint32_t COL_G1 = 256;   // [K;Q] K^T (phasor role -> inverse role)
constexpr uint32_t COL_KQ = 320;   // [NKQ] at 320, 384, 448: [K;Q] bf16 pairs, row r in lane r
constexpr uint32_t TMEM_COLS = 512;
static_assert(COL_KQ + 64 * NKQ <= TMEM_COLS, "tensor memory budget");

__device__ __forceinline__ uint32_t cm_off(int r, int k, int rg) {
  return (uint32_t)((r >> 3) * rg + (k >> 3) * 128 + (r & 7) * 16 + (k & 7) * 2);
}
// V / E tile: column group g = ch / 8 of all 64 tokens is 1 KB (the layout eight TMA
// boxes of 8 channels x 64 tokens produce): byte (ch / 8) * 1024 + t * 16 + (ch % 8) * 2.
__device__ __forceinline__ uint32_t v_off(int t, int ch) { return (uint32_t)((ch >> 3) * 1024 + t * 16 + (ch & 7) * 2); }

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&h);
}

// sin/cos of a phase: reduced to [-pi, pi] (x - 2 pi round(x / 2 pi), the rounding done on
// the FMA pipe by the 1.5 * 2^23 trick, 2 pi split in two parts), then the hardware
// approximation; the error is far below bf16 resolution.
__device__ __forceinline__ void fast_sincos(float x, float *s, float *c) {
  const float k = fmaf(x, 0.15915494309189535f, 12582912.0f) - 12582912.0f;
  float r = fmaf(-k, 6.28318548202514648f, x);
  r = fmaf(-k, -1.7484556e-07f, r);
  __sincosf(r, s, c);
}

// 16-bit operand pairs: bf16 (real beta) or fp16 (complex beta, CB: the isometric update
// does not damp rounding errors, so its tiles keep 10 mantissa bits; the tiles that could
// grow are range-checked, values past 65504 set `over`, reported as DP_ERR_RANGE).
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
__host__ __device__ constexpr uint32_t idesc_op(int M, int N, bool a_mn_major, bool b_mn_major) {
  return F16 ? idesc_f16(M, N, a_mn_major, b_mn_major) : idesc_bf16(M, N, a_mn_major, b_mn_major);
}
// The write key of one fp16 (cos, sin) pair: beta kappa = (br c - bi s, br s + bi c).
__device__ __forceinline__ uint32_t rotate_pair(uint32_t cs, float br, float bi) {
  const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&cs));
  return pack_op<true>(fmaf(br, f.x, -bi * f.y), fmaf(br, f.y, bi * f.x));
}

// The bf16 pair (cos theta, sin theta) of a bf16 phase given as raw bits.  (Measured
// alternatives, all slower on this kernel: the FMA-pipe polynomial poly_sincos for all or
// half of the phases, and a shared-memory table of the bf16 phases.)
template <bool CB>
__device__ __forceinline__ uint32_t phasor_word(uint32_t bits) {
  float s, c;
  fast_sincos(__uint_as_float(bits << 16), &s, &c);
  return pack_op<CB>(c, s);
}

// One warp: D[16 x 16] = X[16 x K] Y[K x 16], X(i, k) = x[i * xs_i + k * xs_k],
// Y(k, j) = y[k * ys_k + j * ys_j] (fp32 in shared memory, tf32 products), returned as
// two m16n8 fragments.
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

struct PipeArgs {
  const void *beta;
  int beta_dt;
  const float *state_in;
  float *out;
  float *state_out;
  int H, L;
  SeqStrides s_b, s_out;
  int *err;
  ChunkMapDims dk, dq, dv, dout;  // map dimension of token, head and batch of each tensor
  int out_tma;                    // outputs by bulk tensor stores through maps.out
};

// theta_k and theta_q with a 64 x 64 box; v with an 8 x 64 box (one column group); out
// with a 32 x 64 box.
struct alignas(64) PipeMaps {
  CUtensorMap tk, tq, v8, out;
};

struct PipeBars {
  uint64_t stage[2];         // theta stage loaded (phasor role)
  uint64_t g1_done;          // G1 complete (MMA commit) -> inverse role
  uint64_t g1_free;          // inverse role done with the G1 accumulator -> phasor role
  uint64_t kq_free[NKQ];     // chain MMAs done with a K / Q slot -> phasor role
  uint64_t bt_full[2];       // bT, P of a chunk written -> chain
  uint64_t bt_free[2];       // chain MMAs done with a bT / P slot -> inverse role
  uint64_t v_full[2];        // V of a chunk loaded -> chain
  uint64_t chain_mma;        // chain MMA completion
  uint64_t out_empty[2];     // outputs of an R3 slot read out of tensor memory -> chain
  uint32_t tmem_base;
  int fail;
  int range;  // a 16-bit tile value out of range (complex beta)
};
static_assert(sizeof(PipeBars) <= 256, "barrier block");

__device__ __forceinline__ void issue_theta_loads(const PipeMaps &m, const PipeArgs &a, uint8_t *stage, uint64_t *bar,
                                                  int c0, int h, int b) {
  mbar_arrive_expect_tx(bar, (uint32_t)STAGE_BYTES);
  tma_load_chunk(stage, &m.tk, a.dk, c0, h, b, bar);
  tma_load_chunk(stage + kC * 128, &m.tq, a.dq, c0, h, b, bar);
}

__device__ __forceinline__ void issue_v_loads(const PipeMaps &m, const PipeArgs &a, uint8_t *vt, uint64_t *bar, int c0,
                                              int h, int b) {
  mbar_arrive_expect_tx(bar, (uint32_t)T64_BYTES);
#pragma unroll
  for (int g = 0; g < 8; ++g) tma_load_colgroup(vt + g * 1024, &m.v8, a.dv, 8 * g, c0, h, b, bar);
}

// Outputs of chunk cc (row t = token, columns 32 hc .. + 31 of the 64 value channels) from
// R3 slot cc & 1 of tensor memory: into the output tile, then two bulk tensor stores issued
// by `lead` (tokens past L are not written); with no output map, straight from registers.
// Run by the four phasor warps of TMEM lane quarters 2 and 3 (barrier BAR_OUT); `lead`
// frees the slot (out_empty) as soon as all four warps hold their rows in registers.
template <bool CB>
__device__ __noinline__ void pipe_store_out(const PipeArgs &a, const PipeMaps &maps, uint8_t *smem, PipeBars *bars,
                                            uint32_t taddr, int t, int hc, bool lead, int cc, int h, int b) {
  // real beta: the accumulator holds 64 O; complex beta: O (its tiles carry the 1 / 64)
  const float scale = CB ? 1.0f : 1.0f / 64.0f;
  const int tt = cc * kC + t;
  float o[32];
  tmem_ld32_sync(taddr, o);
  tc_fence_before();
  if (lead) bulk_wait_read_all();  // the previous chunk's stores have read the tile
  group_sync(BAR_OUT, 128);
  if (lead) mbar_arrive(&bars->out_empty[cc & 1]);
  if (a.out_tma) {
    uint8_t *orow = smem + OFF_OUT + hc * (kC * 128) + t * 128;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      *reinterpret_cast<float4 *>(orow + ((i ^ (t & 7)) << 4)) =
          make_float4(o[4 * i] * scale, o[4 * i + 1] * scale, o[4 * i + 2] * scale, o[4 * i + 3] * scale);
    fence_proxy_async_smem();
    group_sync(BAR_OUT, 128);
    if (lead) {
      tma_store_chunk(&maps.out, a.dout, smem + OFF_OUT, 0, cc * kC, h, b);
      tma_store_chunk(&maps.out, a.dout, smem + OFF_OUT + kC * 128, 32, cc * kC, h, b);
      bulk_commit_group();
    }
  } else if (tt < a.L) {
    float *orow = a.out + b * a.s_out.b + h * a.s_out.h + (int64_t)tt * a.s_out.t + 32 * hc;
#pragma unroll
    for (int i = 0; i < 32; i += 4)
      *reinterpret_cast<float4 *>(orow + i) =
          make_float4(o[i] * scale, o[i + 1] * scale, o[i + 2] * scale, o[i + 3] * scale);
  }
}

// ------------------------------------------------------------------------ phasor role
// Warp w computes half w / 4 (channels 32 (w / 4) ..) of rows 32 (w % 4) .. + 31 of
// [K; Q] (its TMEM lane quarter): row r is K row r for r < 64, Q row r - 64 otherwise,
// from stage row r (theta_k rows, then theta_q rows).  The stage is written by TMA with
// the 128-byte swizzle, so the 32 rows a warp reads at once fall on distinct bank groups.
// Two stages: the phases of chunk c + 1 are in flight while chunk c's are used.
template <bool CB>
__device__ bool phasor_role(const PipeArgs &a, const PipeMaps &maps, uint8_t *smem, PipeBars *bars, uint32_t tmem,
                            int b, int h, int nchunks) {
  const int tid = threadIdx.x, warp = tid >> 5, h2 = warp >> 2;
  const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
  const int L = a.L;
  const int r = (warp & 3) * 32 + (tid & 31), t = r & 63;
  const bool is_k = r < kC;
  int issued = 0, consumed = 0, g1_issued = 0;
  bool ok = true;
  // complex beta: phi of this thread's K row, a chunk ahead (raw bits)
  const int64_t pbase = b * a.s_b.b + h * a.s_b.h;
  uint32_t phi_next = 0u;
  if (CB && is_k && t < L) phi_next = load_raw_scalar(a.beta, a.beta_dt, pbase + (int64_t)t * a.s_b.t);
  for (int k = 0; k < 2 && k < nchunks; ++k) {
    if (tid == 0) issue_theta_loads(maps, a, smem + OFF_STAGE + k * STAGE_BYTES, &bars->stage[k], k * kC, h, b);
    issued = k + 1;
  }
  // Iteration c makes the phasors of chunk c and, once the chain has finished chunk
  // c - NKQ (kq_free: its last MMA, G5, has completed), stores that chunk's outputs; NKQ
  // more iterations after the last chunk store the remaining outputs.
  for (int c = 0; c < nchunks + NKQ; ++c) {
    const int ks = c % NKQ, t0 = c * kC, nvalid = min(kC, L - t0), sb = c & 1;
    uint8_t *kt = smem + OFF_K + ks * K_BYTES;
    uint8_t *stage = smem + OFF_STAGE + sb * STAGE_BYTES;
    const uint8_t *srow = stage + r * 128;
    const bool work = c < nchunks;
    if (tid == 0) {
      if (c >= NKQ) ok = mbar_wait(&bars->kq_free[ks], (uint32_t)((c / NKQ - 1) & 1), kTimeoutNs);
      if (ok && work) ok = mbar_wait(&bars->stage[sb], (uint32_t)((c >> 1) & 1), kTimeoutNs);
    }
    if (group_any(!ok, BAR_PH, kPhThreads)) { ok = false; break; }
    if (c >= NKQ && (warp & 3) >= 2) {
      const int cc = c - NKQ;
      pipe_store_out<CB>(a, maps, smem, bars, tmem + lane_base + COL_R3 + 64 * (cc & 1) + 32 * h2,
                     ((warp & 3) - 2) * 32 + (tid & 31), h2, tid == 64, cc, h, b);
    }
    if (!work) continue;
    consumed = c + 1;
    // rows past L hold zero phasors.  The phasors are computed unconditionally and masked
    // afterwards: a per-phasor select around the sincos makes the compiler branch around
    // each one, which serialises them (twice the time of this loop, measured).
    const uint32_t vmask = t < nvalid ? 0xFFFFFFFFu : 0u;
    float br = 1.f, bi = 0.f;  // complex beta of this K row: 1 + e^{i phi}
    if (CB) {
      const uint32_t phi_cur = phi_next;
      phi_next = 0u;
      if (is_k && t0 + kC + t < L) phi_next = load_raw_scalar(a.beta, a.beta_dt, pbase + (int64_t)(t0 + kC + t) * a.s_b.t);
      fast_sincos(raw_scalar_to_f32(phi_cur, a.beta_dt), &bi, &br);
      br += 1.f;
    }
    {
      uint32_t w[32];
#pragma unroll
      for (int s4 = 0; s4 < 4; ++s4) {
        const int sg = 4 * h2 + s4;  // 16-byte chunk of the row: channels 8 sg .. 8 sg + 7
        const uint4 raw = *reinterpret_cast<const uint4 *>(srow + ((sg ^ (r & 7)) << 4));
        const uint32_t rw[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          w[8 * s4 + 2 * i] = phasor_word<CB>(rw[i] & 0xFFFFu) & vmask;
          w[8 * s4 + 2 * i + 1] = phasor_word<CB>(rw[i] >> 16) & vmask;
        }
      }
      tmem_st32(tmem + lane_base + COL_KQ + 64 * ks + 32 * h2, w);
      if (is_k) {
        // the K row (complex beta: the write key W = beta K) also into the shared-memory
        // tile: features 64 h2 + 8 g .. (4 channels)
#pragma unroll
        for (int g = 0; g < 8; ++g) {
          uint4 x = make_uint4(w[4 * g], w[4 * g + 1], w[4 * g + 2], w[4 * g + 3]);
          if (CB)
            x = make_uint4(rotate_pair(x.x, br, bi), rotate_pair(x.y, br, bi), rotate_pair(x.z, br, bi),
                           rotate_pair(x.w, br, bi));
          *reinterpret_cast<uint4 *>(kt + cm_off(t, 64 * h2 + 8 * g, RG_KQ)) = x;
        }
      }
    }
    tmem_st_wait();
    fence_proxy_async_smem();
    tc_fence_before();
    group_sync(BAR_PH, kPhThreads);
    if (warp == 0) {
      // the stage is free: the phases of chunk c + 2; then G1 = [K; Q] K^T (A from TMEM)
      if (tid == 0) {
        if (c + 2 < nchunks) {
          issue_theta_loads(maps, a, stage, &bars->stage[sb], t0 + 2 * kC, h, b);
          issued = c + 3;
        }
        if (c >= 1) ok = mbar_wait(&bars->g1_free, (uint32_t)((c - 1) & 1), kTimeoutNs);
      }
      ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
      if (ok) {
        tc_fence_after();
        const uint32_t sk = smem_u32(kt);
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_f16_ts(tmem + COL_G1, tmem + COL_KQ + 64 * ks + 8 * kk, make_desc(sk + kk * 256, 128, RG_KQ),
                       idesc_op<CB>(128, 64, false, false), kk > 0);
          mma_commit(&bars->g1_done);
        }
        __syncwarp();
        g1_issued = c + 1;
      }
    }
    if (group_any(!ok, BAR_PH, kPhThreads)) { ok = false; break; }
  }
  if (!ok && tid == 0) {
    // let this role's own copies and MMAs land before shared / tensor memory is released
    for (int k = consumed; k < issued; ++k) mbar_wait(&bars->stage[k & 1], (uint32_t)((k >> 1) & 1), kTimeoutNs);
    if (g1_issued > 0) mbar_wait(&bars->g1_done, (uint32_t)((g1_issued - 1) & 1), kTimeoutNs);
  }
  if (tid == 64 && a.out_tma) bulk_wait_all();  // the output stores are complete
  return ok;
}

// ----------------------------------------------------------------------- inverse role
template <bool CB>
__device__ bool inverse_role(const PipeArgs &a, uint8_t *smem, PipeBars *bars, uint32_t tmem, int b, int h,
                             int nchunks) {
  const int itid = threadIdx.x - kInvBase, iw = itid >> 5, lane = itid & 31;  // iw = TMEM lane quarter
  const uint32_t lane_base = (uint32_t)(iw * 32) << 16;
  const int L = a.L;
  float *at = reinterpret_cast<float *>(smem + OFF_AT);
  float *tf = reinterpret_cast<float *>(smem + OFF_TF);
  float *zs = reinterpret_cast<float *>(smem + OFF_Z);
  float *bs = reinterpret_cast<float *>(smem + OFF_BETA);
  const float inv64 = 1.0f / 64.0f;
  const int64_t bbase = b * a.s_b.b + h * a.s_b.h;
  bool ok = true, over = false;
  uint32_t bnext = 0u;  // raw bits of the next chunk's beta (converted when used)
  if (!CB && itid < kC && itid < L) bnext = load_raw_scalar(a.beta, a.beta_dt, bbase + (int64_t)itid * a.s_b.t);
  for (int c = 0; c < nchunks; ++c) {
    const int gs = c & 1, t0 = c * kC;
    uint8_t *pb = smem + OFF_P + gs * T64_BYTES;
    uint8_t *btb = smem + OFF_BT + gs * T64_BYTES;
    if (itid < kC) bs[itid] = raw_scalar_to_f32(bnext, a.beta_dt);
    bnext = 0u;
    if (!CB && itid < kC && t0 + kC + itid < L)
      bnext = load_raw_scalar(a.beta, a.beta_dt, bbase + (int64_t)(t0 + kC + itid) * a.s_b.t);
    if (itid == 0) {
      ok = mbar_wait(&bars->g1_done, (uint32_t)(c & 1), kTimeoutNs);
      if (ok && c >= 2) ok = mbar_wait(&bars->bt_free[gs], (uint32_t)(((c - 2) >> 1) & 1), kTimeoutNs);
    }
    if (group_any(!ok, BAR_INV, kInvThreads)) { ok = false; break; }
    tc_fence_after();

    // ---- A^T from the (exactly symmetric) Gram rows, At[k][i] = beta_k G[k][i] / 64 for
    //      i > k (quarters 0, 1); P = tril(Q K^T) in bf16 (quarters 2, 3)
    if (CB && iw < 2) {
      // row i of K W^T: A[i][k] = G1[i][k] / 64 for k < i (not symmetric), stored as column
      // i of A^T
      const int i = iw * 32 + lane;
#pragma unroll 1
      for (int hf = 0; hf < 2; ++hf) {
        float g[32];
        tmem_ld32_sync(tmem + lane_base + COL_G1 + 32 * hf, g);
#pragma unroll
        for (int kk = 0; kk < 32; ++kk) at[(32 * hf + kk) * LDA + i] = (32 * hf + kk < i) ? g[kk] * inv64 : 0.f;
      }
    } else if (iw < 2) {
      const int k = iw * 32 + lane;
      const float bk = bs[k] * inv64;
#pragma unroll 1
      for (int hf = 0; hf < 2; ++hf) {
        float g[32];
        tmem_ld32_sync(tmem + lane_base + COL_G1 + 32 * hf, g);
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
      }
    } else {
      const int t = (iw - 2) * 32 + lane;
#pragma unroll 1
      for (int hf = 0; hf < 2; ++hf) {
        float p[32];
        tmem_ld32_sync(tmem + lane_base + COL_G1 + 32 * hf, p);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int s = 32 * hf + 8 * u;
          const float *pp = p + 8 * u;
          uint4 w;
          const float ps = CB ? inv64 : 1.f;  // fp16 tiles hold P / 64
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
    group_sync(BAR_INV, kInvThreads);
    if (itid == 0) mbar_arrive(&bars->g1_free);  // the G1 accumulator has been read

    // ---- 16 x 16 diagonal blocks of (I + A)^-1: right-looking substitution, the column in
    //      registers (threads 0..63: block itid / 16, column itid % 16), the next row of
    //      A^T loaded while the current one is applied
    if (itid < 64) {
      const int o = 16 * (itid >> 4), col = itid & 15;
      float cl[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) cl[i] = (i == col) ? 1.f : 0.f;
      float nx[16];
#pragma unroll
      for (int i4 = 0; i4 < 16; i4 += 4) {
        const float4 v = *reinterpret_cast<const float4 *>(at + o * LDA + o + i4);
        nx[i4] = v.x; nx[i4 + 1] = v.y; nx[i4 + 2] = v.z; nx[i4 + 3] = v.w;
      }
#pragma unroll
      for (int k = 0; k < 15; ++k) {
        float cur[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) cur[i] = nx[i];
        if (k + 1 < 15) {
#pragma unroll
          for (int i4 = ((k + 2) & ~3); i4 < 16; i4 += 4) {
            const float4 v = *reinterpret_cast<const float4 *>(at + (o + k + 1) * LDA + o + i4);
            nx[i4] = v.x; nx[i4 + 1] = v.y; nx[i4 + 2] = v.z; nx[i4 + 3] = v.w;
          }
        }
        const float tk = cl[k];
#pragma unroll
        for (int i = k + 1; i < 16; ++i) cl[i] = fmaf(-cur[i], tk, cl[i]);
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) tf[(o + i) * LDA + o + col] = cl[i];
    }
    group_sync(BAR_INV, kInvThreads);

    // ---- 16 -> 32 merge of block pairs (0,1), (2,3) on warps 0, 1 (tf32 MMA):
    //      Z = A[16+i][k] T[k][j], then T[16+i][j] = -T11 Z
    if (iw < 2) {
      const int o = 32 * iw;
      float d0[4], d1[4];
      warp_gemm16<16>(d0, d1, at + o * LDA + o + 16, 1, LDA, tf + o * LDA + o, LDA, 1, lane);
      warp_store16(zs + 16 * iw * LDZ, LDZ, d0, d1, 1.f, lane);
      __syncwarp();
      warp_gemm16<16>(d0, d1, tf + (o + 16) * LDA + o + 16, LDA, 1, zs + 16 * iw * LDZ, LDZ, 1, lane);
      warp_store16(tf + (o + 16) * LDA + o, LDA, d0, d1, -1.f, lane);
    }
    group_sync(BAR_INV, kInvThreads);

    // ---- 32 -> 64 merge: Z = A10 T00 (A10[i][k] = At[k][32 + i]), T[32+i][j] = -T11 Z;
    //      one 16 x 16 tile per warp
    {
      const int mi = 16 * (iw >> 1), nj = 16 * (iw & 1);
      float d0[4], d1[4];
      warp_gemm16<32>(d0, d1, at + 32 + mi, 1, LDA, tf + nj, LDA, 1, lane);
      warp_store16(zs + mi * LDZ + nj, LDZ, d0, d1, 1.f, lane);
      group_sync(BAR_INV, kInvThreads);
      warp_gemm16<32>(d0, d1, tf + (32 + mi) * LDA + 32, LDA, 1, zs + nj, LDZ, 1, lane);
      warp_store16(tf + (32 + mi) * LDA + nj, LDA, d0, d1, -1.f, lane);
    }
    group_sync(BAR_INV, kInvThreads);

    // ---- bT = diag(beta) T -> bf16 (row i = itid % 64, columns 32 (itid / 64) ..: eight
    //      consecutive rows per quarter warp, so the row loads and tile stores do not conflict)
    {
      const int i = itid & 63, c0 = 32 * (itid >> 6);
      const float bi = CB ? 1.f : bs[i];  // complex beta: U = T E
      const float *tr = tf + i * LDA + c0;
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) {
        const float4 x0 = *reinterpret_cast<const float4 *>(tr + 8 * c8);
        const float4 x1 = *reinterpret_cast<const float4 *>(tr + 8 * c8 + 4);
        *reinterpret_cast<uint4 *>(btb + cm_off(i, c0 + 8 * c8, RG_64)) =
            make_uint4(pack_chk<CB>(bi * x0.x, bi * x0.y, over), pack_chk<CB>(bi * x0.z, bi * x0.w, over),
                       pack_chk<CB>(bi * x1.x, bi * x1.y, over), pack_chk<CB>(bi * x1.z, bi * x1.w, over));
      }
    }
    fence_proxy_async_smem();
    group_sync(BAR_INV, kInvThreads);
    if (itid == 0) mbar_arrive(&bars->bt_full[gs]);
  }
  if (CB && over) atomicOr(&bars->range, 1);
  return ok;
}

// ------------------------------------------------------------------------- chain role
// Warp cw (0..7) of the role: TMEM lane quarter q = cw % 4, column half hc = cw / 4.
template <bool CB>
__device__ bool chain_role(const PipeArgs &a, const PipeMaps &maps, uint8_t *smem, PipeBars *bars, uint32_t tmem,
                           int bh, int b, int h, int nchunks) {
  const int ctid = threadIdx.x - kChBase, cw = ctid >> 5, lane = ctid & 31;
  const int q = cw & 3, hc = cw >> 2;
  const uint32_t lane_base = (uint32_t)(q * 32) << 16;
  uint8_t *ub = smem + OFF_U;
  uint8_t *s0 = smem + OFF_S0;
  const float inv64 = 1.0f / 64.0f;
  const int64_t sbase = (int64_t)bh * kDv * kF;
  const int j = q * 32 + lane;  // feature row of S^T in C1

  // initial state^T -> TMEM (row j, value channels 32 hc ..)
  {
    float vals[16];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        vals[i] = a.state_in ? a.state_in[sbase + (int64_t)(32 * hc + 16 * u + i) * kF + j] : 0.f;
      tmem_st16(tmem + lane_base + COL_S + 32 * hc + 16 * u, vals);
    }
  }
  tmem_st_wait();
  tc_fence_before();
  group_sync(BAR_CH, kChThreads);

  // Thread 32 (warp 1) is the role's input thread: it issues the V loads and waits for the
  // next chunk's bT / P and V while thread 0 issues and waits for this chunk's state MMAs,
  // so the chain never starts a chunk with those waits.
  const bool in_thread = ctid == 32;
  uint32_t cm_phase = 0;
  int v_issued = 0, v_consumed = 0, cm_pending = 0;
  bool ok = true, over = false;
  // complex beta: the S^T operand holds S^T / 64 (fp16 range), so G3 yields K S^T / 64
  const float ss64 = CB ? 1.0f / 64.0f : 1.0f;
  if (in_thread) {
    for (int k = 0; k < 2 && k < nchunks; ++k) {
      issue_v_loads(maps, a, smem + OFF_V + k * T64_BYTES, &bars->v_full[k], k * kC, h, b);
      v_issued = k + 1;
    }
    if (nchunks > 0) {
      ok = mbar_wait(&bars->bt_full[0], 0u, kTimeoutNs);
      if (ok) ok = mbar_wait(&bars->v_full[0], 0u, kTimeoutNs);
    }
  }

  // thread 0 (the lane elect_one picks in warp 0): wait for the MMAs committed last
  auto mma_wait = [&]() {
    ++cm_pending;
    const bool r = mbar_wait(&bars->chain_mma, cm_phase, kTimeoutNs);
    if (r) {
      cm_phase ^= 1;
      --cm_pending;
    }
    return r;
  };

  for (int c = 0; c < nchunks; ++c) {
    const int gs = c & 1, ks = c % NKQ;
    uint8_t *kt = smem + OFF_K + ks * K_BYTES;
    uint8_t *vt = smem + OFF_V + gs * T64_BYTES;
    uint8_t *btb = smem + OFF_BT + gs * T64_BYTES;
    uint8_t *pb = smem + OFF_P + gs * T64_BYTES;
    const uint32_t r3 = COL_R3 + 64 * gs;

    // bT / P and V of chunk c are present; S^T holds the state at its start
    if (group_any(!ok, BAR_CH, kChThreads)) { ok = false; break; }
    v_consumed = c + 1;
    tc_fence_after();

    // ---- C1: S^T (fp32, TMEM) -> bf16 operand tile (row j, columns 32 hc ..)
    {
      float sv[32];
      tmem_ld32_sync(tmem + lane_base + COL_S + 32 * hc, sv);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float *ss = sv + 8 * u;
        *reinterpret_cast<uint4 *>(s0 + cm_off(j, 32 * hc + 8 * u, RG_64)) =
            make_uint4(pack_chk<CB>(ss[0] * ss64, ss[1] * ss64, over), pack_chk<CB>(ss[2] * ss64, ss[3] * ss64, over),
                       pack_chk<CB>(ss[4] * ss64, ss[5] * ss64, over), pack_chk<CB>(ss[6] * ss64, ss[7] * ss64, over));
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    group_sync(BAR_CH, kChThreads);

    // ---- C2: G3 = [K; Q] S^T -> R3 slot (M = 128, N = 64, K = 128)
    if (cw == 0) {
      tc_fence_after();
      const uint32_t ss = smem_u32(s0);
      if (elect_one()) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          mma_f16_ts(tmem + r3, tmem + COL_KQ + 64 * ks + 8 * kk, make_desc(ss + kk * 2 * RG_64, RG_64, 128),
                     idesc_op<CB>(128, 64, false, true), kk > 0);
        mma_commit(&bars->chain_mma);
      }
      __syncwarp();
      if (lane == 0) ok = mma_wait();
    }
    if (group_any(!ok, BAR_CH, kChThreads)) { ok = false; break; }
    tc_fence_after();

    // ---- C3: E = V - K S^T / 64 -> bf16 in place of V (row t = lane of quarters 0, 1)
    if (q < 2) {
      const int t = q * 32 + lane;
      float ks[32];
      tmem_ld32_sync(tmem + lane_base + r3 + 32 * hc, ks);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        uint4 *vp = reinterpret_cast<uint4 *>(vt + v_off(t, 32 * hc + 8 * u));
        const uint4 vr = *vp;
        const uint32_t vw[4] = {vr.x, vr.y, vr.z, vr.w};
        uint32_t ew[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 vv = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&vw[i]));
          if (CB)  // the state-read rows already carry the 1 / 64
            ew[i] = pack_chk<true>(vv.x - ks[8 * u + 2 * i], vv.y - ks[8 * u + 2 * i + 1], over);
          else
            ew[i] = pack_bf16(vv.x - ks[8 * u + 2 * i] * inv64, vv.y - ks[8 * u + 2 * i + 1] * inv64);
        }
        *vp = make_uint4(ew[0], ew[1], ew[2], ew[3]);
      }
      fence_proxy_async_smem();
    }
    tc_fence_before();
    group_sync(BAR_CH, kChThreads);

    // ---- C3u: U = bT E (M = 64, N = 64, K = 64) -> RU.  E's tile is column-group-major:
    //      along K (tokens) 8-row core matrices are 128 bytes apart, along N 1 KB.
    if (cw == 0) {
      tc_fence_after();
      const uint32_t sb = smem_u32(btb), se = smem_u32(vt);
      if (elect_one()) {
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f16_ss(tmem + COL_RU, make_desc(sb + kk * 256, 128, RG_64), make_desc(se + kk * 256, 128, 1024),
                     idesc_op<CB>(64, 64, false, true), kk > 0);
        mma_commit(&bars->chain_mma);
      }
      __syncwarp();
      if (lane == 0) ok = mma_wait();
    }
    if (group_any(!ok, BAR_CH, kChThreads)) { ok = false; break; }
    tc_fence_after();

    // ---- C3c: U -> bf16 operand tile (M = 64 rows: row 16 q + lane in lanes < 16)
    {
      const int t = 16 * q + lane;
      float uv[32];
      tmem_ld32_sync(tmem + lane_base + COL_RU + 32 * hc, uv);
      if (lane < 16) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float *uu = uv + 8 * u;
          *reinterpret_cast<uint4 *>(ub + cm_off(t, 32 * hc + 8 * u, RG_64)) =
              make_uint4(pack_chk<CB>(uu[0], uu[1], over), pack_chk<CB>(uu[2], uu[3], over),
                         pack_chk<CB>(uu[4], uu[5], over), pack_chk<CB>(uu[6], uu[7], over));
        }
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    group_sync(BAR_CH, kChThreads);

    // ---- C4: G4 S^T += K^T U (M = 128), committed and waited for on its own (the next chunk
    //      needs only the state), then G5 R3 += [X; P] U (M = 128, A starting 8 KB before P:
    //      rows 64.. of R3 (Q S^T) gain P U, rows 0.. (K S^T, used) are don't-care).  The
    //      commits after G5 free this chunk's K / Q and bT / P slots.
    if (cw == 0) {
      tc_fence_after();
      const uint32_t sk = smem_u32(kt), su = smem_u32(ub), sp = smem_u32(pb) - 8 * RG_64;
      if (elect_one()) {
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f16_ss(tmem + COL_S, make_desc(sk + kk * 2 * RG_KQ, RG_KQ, 128),
                     make_desc(su + kk * 2 * RG_64, RG_64, 128), idesc_op<CB>(128, 64, true, true), 1u);
        mma_commit(&bars->chain_mma);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f16_ss(tmem + r3, make_desc(sp + kk * 256, 128, RG_64), make_desc(su + kk * 2 * RG_64, RG_64, 128),
                     idesc_op<CB>(128, 64, false, true), 1u);
        mma_commit(&bars->kq_free[ks]);
        mma_commit(&bars->bt_free[gs]);
      }
      __syncwarp();
      if (lane == 0) ok = mma_wait();
    } else if (in_thread) {
      // V of chunk c + 2 into this chunk's slot (its last reader, U of chunk c, is done);
      // then the inputs of chunk c + 1
      if (c + 2 < nchunks) {
        issue_v_loads(maps, a, vt, &bars->v_full[gs], (c + 2) * kC, h, b);
        v_issued = c + 3;
      }
      if (c + 1 < nchunks) {
        ok = mbar_wait(&bars->bt_full[gs ^ 1], (uint32_t)(((c + 1) >> 1) & 1), kTimeoutNs);
        if (ok) ok = mbar_wait(&bars->v_full[gs ^ 1], (uint32_t)(((c + 1) >> 1) & 1), kTimeoutNs);
        // R3 slot of chunk c + 1: the outputs of chunk c - 1 have been read out of it
        if (ok && c >= 1) ok = mbar_wait(&bars->out_empty[gs ^ 1], (uint32_t)(((c - 1) >> 1) & 1), kTimeoutNs);
      }
    }
  }

  if (ok) {
    // the last chunk's state update (G4) has completed (thread 0's wait)
    if (group_any(!ok, BAR_CH, kChThreads)) ok = false;
    tc_fence_after();
  }
  if (ok) {
    // final state: TMEM S^T -> complex64 state (row o, interleaved column j)
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      float sv[16];
      tmem_ld16(tmem + lane_base + COL_S + 32 * hc + 16 * u, sv);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 16; ++i) a.state_out[sbase + (int64_t)(32 * hc + 16 * u + i) * kF + j] = sv[i];
    }
  } else if (ctid == 0) {
    // let this role's MMAs finish before shared and tensor memory are released
    mma_commit(&bars->chain_mma);  // arrives once every MMA issued so far has completed
    for (int k = 0; k <= cm_pending; ++k) {
      if (!mbar_wait(&bars->chain_mma, cm_phase, kTimeoutNs)) break;
      cm_phase ^= 1;
    }
  } else if (in_thread) {
    for (int k = v_consumed; k < v_issued; ++k) mbar_wait(&bars->v_full[k & 1], (uint32_t)((k >> 1) & 1), kTimeoutNs);
  }
  if (CB && over) atomicOr(&bars->range, 1);
  return ok;
}

template <bool CB>
__global__ void __launch_bounds__(kThreads, 1) core_pipe_kernel(const __grid_constant__ PipeArgs a,
                                                                 const __grid_constant__ PipeMaps maps) {
  extern __shared__ __align__(1024) uint8_t smem[];
  PipeBars *bars = reinterpret_cast<PipeBars *>(smem + OFF_BAR);
  float *tf = reinterpret_cast<float *>(smem + OFF_TF);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int bh = blockIdx.x, b = bh / a.H, h = bh % a.H;
  const int nchunks = (a.L + kC - 1) / kC;

  if (tid == 0) {
    mbar_init(&bars->stage[0], 1);
    mbar_init(&bars->stage[1], 1);
    mbar_init(&bars->g1_done, 1);
    mbar_init(&bars->g1_free, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->bt_full[i], 1);
      mbar_init(&bars->bt_free[i], 1);
      mbar_init(&bars->v_full[i], 1);
    }
    for (int i = 0; i < NKQ; ++i) mbar_init(&bars->kq_free[i], 1);
    mbar_init(&bars->chain_mma, 1);
    mbar_init(&bars->out_empty[0], 1);
    mbar_init(&bars->out_empty[1], 1);
    bars->fail = 0;
    bars->range = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&bars->tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  // T's strictly upper blocks are never written: zero them once
  for (int i = tid; i < kC * LDA; i += kThreads) tf[i] = 0.f;
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  bool ok;
  if (tid < kInvBase)
    ok = phasor_role<CB>(a, maps, smem, bars, tmem, b, h, nchunks);
  else if (tid < kChBase)
    ok = inverse_role<CB>(a, smem, bars, tmem, b, h, nchunks);
  else
    ok = chain_role<CB>(a, maps, smem, bars, tmem, bh, b, h, nchunks);
  if (!ok) atomicExch(&bars->fail, 1);

  tc_fence_before();
  __syncthreads();
  if (tid == 0 && bars->fail) atomicCAS(a.err, 0, DP_ERR_TIMEOUT);
  if (CB && tid == 0 && bars->range) atomicCAS(a.err, 0, DP_ERR_RANGE);
  if (warp == 0) tmem_dealloc(tmem, TMEM_COLS);
}

}  // namespace

// The pipelined kernel for dp_core_fwd (real beta) and dp_core_cbeta_fwd (cbeta: `beta`
// holds phi of the complex beta 1 + e^{i phi}) when its tensor maps encode (L >= 64);
// returns false without launching otherwise (the caller then runs core_fwd_tc).
bool core_fwd_pipe(const void *tk, const void *tq, const void *v, const void *beta, int beta_dt,
                   const float *state_in, float *out, float *state_out, int B, int H, int L, const SeqStrides *s,
                   cudaStream_t stream, bool cbeta, int *rc) {
  if (L < kC) return false;
  PipeArgs a;
  memset(&a, 0, sizeof(a));
  a.beta = beta;
  a.beta_dt = beta_dt;
  a.state_in = state_in;
  a.out = out;
  a.state_out = state_out;
  a.H = H;
  a.L = L;
  a.s_b = s[3];
  a.s_out = s[4];
  a.err = device_error_ptr();
  if (!a.err) {
    *rc = set_error(DP_ERR_CUDA, "core_fwd_pipe: device error word unavailable");
    return true;
  }
  PipeMaps maps;
  memset(&maps, 0, sizeof(maps));
  if (!encode_chunk_map(&maps.tk, &a.dk, tk, B, H, L, s[0], 64, true) ||
      !encode_chunk_map(&maps.tq, &a.dq, tq, B, H, L, s[1], 64, true) ||
      !encode_chunk_map(&maps.v8, &a.dv, v, B, H, L, s[2], 8))
    return false;
  a.out_tma = encode_out_map(&maps.out, &a.dout, out, B, H, L, s[4]) ? 1 : 0;
  auto kern = cbeta ? core_pipe_kernel<true> : core_pipe_kernel<false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  if (e != cudaSuccess) {
    *rc = set_error(DP_ERR_CUDA, std::string("core_pipe smem attr: ") + cudaGetErrorString(e));
    return true;
  }
  kern<<<B * H, kThreads, SMEM_BYTES, stream>>>(a, maps);
  *rc = check_launch("core_pipe_kernel");
  return true;
}

}  // namespace dp
