// Single-token decode step of the complex delta rule (memory-bound state update).
//
// Reference: DeltaPhaseHolographicBlock.step (delta_phase/layers.py:279-285):
//   v_old = Re(M conj(k)) / D;  M <- M + beta (v - v_old) k^T;  out = Re(M conj(q)) / D
// (the readout uses the updated state).  Same contract as the never-launched
// _triton_streaming_step_kernel (delta_phase/kernels/triton_chunk_delta.py:125-185),
// but on the interleaved complex64 state, so torch's complex tensor is used as is.
//
// Complex beta (ComplexBetaDeltaPhaseBlock.step, layers.py:402-407): beta = 1 + e^{i phi}
// and M <- M + beta (v - v_old) k^T, i.e. the update writes along the rotated key
// w = beta k = (br c - bi s) + i (br s + bi c) per channel (template flag CB, `beta` = phi).
//
// One CTA per (batch, head); one warp per state row (value channel) at a time.  Each
// row is read once and written once with 16-byte accesses (two complex entries per
// lane), so the kernel moves the 2 * Dv * D * 8 bytes of state plus the inputs.
#include "dp_common.cuh"

namespace dp {
namespace {

constexpr int kDecThreads = 256;

__device__ __forceinline__ float load_any(const void *p, int dt, int64_t i) {
  if (dt == DP_F32) return static_cast<const float *>(p)[i];
  if (dt == DP_BF16) return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
  return __half2float(static_cast<const __half *>(p)[i]);
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// The write gate from its raw value: 2 sigmoid(g) for DP_GATE_SIGMOID2 (layers.py:265),
// the value itself otherwise (beta, phi, or the 1 the caller loaded for DP_GATE_ONE).
__device__ __forceinline__ float gate_beta(float g, int gate_mode) {
  return gate_mode == DP_GATE_SIGMOID2 ? 2.f / (1.f + expf(-g)) : g;
}

// kq: smem (4 x D): cos k, sin k, cos q, sin q; CB adds the write key (2 x D).
template <bool kVec4, bool CB>
__global__ void __launch_bounds__(kDecThreads)
decode_kernel(const float *state_in, float *state_out, const void *tk,
              const void *tq, const void *v,
              const void *beta, int in_dt, int beta_dt, int gate_mode,
              float *__restrict__ out, int H, int D, int Dv, SeqStrides s_tk, SeqStrides s_tq, SeqStrides s_v,
              SeqStrides s_b, SeqStrides s_out) {
  extern __shared__ float kq[];
  pdl_wait();
  pdl_trigger();
  const int bh = blockIdx.x, b = bh / H, h = bh % H;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int c = tid; c < D; c += kDecThreads) {
    float s, co;
    sincosf(load_any(tk, in_dt, b * s_tk.b + h * s_tk.h + c), &s, &co);
    kq[c] = co;
    kq[D + c] = s;
    sincosf(load_any(tq, in_dt, b * s_tq.b + h * s_tq.h + c), &s, &co);
    kq[2 * D + c] = co;
    kq[3 * D + c] = s;
  }
  const float inv_d = 1.0f / (float)D;
  const float bt_raw = gate_mode == DP_GATE_ONE ? 1.f : load_any(beta, beta_dt, b * s_b.b + h * s_b.h);
  float bt = gate_beta(bt_raw, gate_mode);
  // write key: the read key (real beta) or beta k (complex beta, then bt = 1)
  const float *wc = kq, *ws = kq + D;
  if (CB) {
    float sp, cp;
    sincosf(bt, &sp, &cp);
    const float br = 1.f + cp;
    __syncthreads();
    for (int c = threadIdx.x; c < D; c += kDecThreads) {
      kq[4 * D + c] = fmaf(br, kq[c], -sp * kq[D + c]);
      kq[5 * D + c] = fmaf(br, kq[D + c], sp * kq[c]);
    }
    wc = kq + 4 * D;
    ws = kq + 5 * D;
    bt = 1.f;
  }
  __syncthreads();
  const int64_t base = (int64_t)bh * Dv * 2 * D;
  for (int o = warp; o < Dv; o += kDecThreads / 32) {
    const float *row_in = state_in + base + (int64_t)o * 2 * D;
    float *row_out = state_out + base + (int64_t)o * 2 * D;
    const float vo = load_any(v, in_dt, b * s_v.b + h * s_v.h + o);
    if (kVec4) {  // two complex entries per lane per step; D % 2 == 0, 16-byte aligned rows
      const int npair = D / 2;
      float4 m[4];
      int cnt = 0;
      float acc = 0.f;
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        const int p = lane + 32 * it;
        if (p < npair) {
          m[it] = reinterpret_cast<const float4 *>(row_in)[p];
          acc += m[it].x * kq[2 * p] + m[it].y * kq[D + 2 * p] + m[it].z * kq[2 * p + 1] +
                 m[it].w * kq[D + 2 * p + 1];
          cnt = it + 1;
        }
      }
      // rows with D > 256 continue in a tail loop (rare shapes)
      for (int p = lane + 128; p < npair; p += 32) {
        float4 t = reinterpret_cast<const float4 *>(row_in)[p];
        acc += t.x * kq[2 * p] + t.y * kq[D + 2 * p] + t.z * kq[2 * p + 1] + t.w * kq[D + 2 * p + 1];
      }
      const float e = bt * (vo - warp_sum(acc) * inv_d);
      float r = 0.f;
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        const int p = lane + 32 * it;
        if (it < cnt && p < npair) {
          float4 t = m[it];
          t.x = fmaf(e, wc[2 * p], t.x);
          t.y = fmaf(e, ws[2 * p], t.y);
          t.z = fmaf(e, wc[2 * p + 1], t.z);
          t.w = fmaf(e, ws[2 * p + 1], t.w);
          reinterpret_cast<float4 *>(row_out)[p] = t;
          r += t.x * kq[2 * D + 2 * p] + t.y * kq[3 * D + 2 * p] + t.z * kq[2 * D + 2 * p + 1] +
               t.w * kq[3 * D + 2 * p + 1];
        }
      }
      for (int p = lane + 128; p < npair; p += 32) {
        float4 t = reinterpret_cast<const float4 *>(row_in)[p];
        t.x = fmaf(e, wc[2 * p], t.x);
        t.y = fmaf(e, ws[2 * p], t.y);
        t.z = fmaf(e, wc[2 * p + 1], t.z);
        t.w = fmaf(e, ws[2 * p + 1], t.w);
        reinterpret_cast<float4 *>(row_out)[p] = t;
        r += t.x * kq[2 * D + 2 * p] + t.y * kq[3 * D + 2 * p] + t.z * kq[2 * D + 2 * p + 1] +
             t.w * kq[3 * D + 2 * p + 1];
      }
      r = warp_sum(r);
      if (lane == 0) out[b * s_out.b + h * s_out.h + o] = r * inv_d;
    } else {  // generic: one complex entry per lane per step
      float acc = 0.f;
      for (int c = lane; c < D; c += 32) {
        const float2 m = reinterpret_cast<const float2 *>(row_in)[c];
        acc += m.x * kq[c] + m.y * kq[D + c];
      }
      const float e = bt * (vo - warp_sum(acc) * inv_d);
      __syncwarp();
      float r = 0.f;
      for (int c = lane; c < D; c += 32) {
        float2 m = reinterpret_cast<const float2 *>(row_in)[c];
        m.x = fmaf(e, wc[c], m.x);
        m.y = fmaf(e, ws[c], m.y);
        reinterpret_cast<float2 *>(row_out)[c] = m;
        r += m.x * kq[2 * D + c] + m.y * kq[3 * D + c];
      }
      r = warp_sum(r);
      if (lane == 0) out[b * s_out.b + h * s_out.h + o] = r * inv_d;
    }
  }
}

// Fast path for even D <= 64 (one float4 = two complex entries per lane and row) and
// Dv <= 8 RPW: warp w owns rows w, w + 8, ...; all of its rows are loaded before any
// reduction, so every lane keeps RPW independent 16-byte loads in flight.
template <int RPW, bool CB>
__global__ void __launch_bounds__(kDecThreads)
decode_rows_kernel(const float *state_in, float *state_out, const void *tk,
                   const void *tq, const void *v,
                   const void *beta, int in_dt, int beta_dt, int gate_mode,
                   float *__restrict__ out, int H, int D, int Dv, SeqStrides s_tk, SeqStrides s_tq, SeqStrides s_v, SeqStrides s_b,
                   SeqStrides s_out) {
  // this (b, h)'s state does not come from the kernels this one overlaps: fetch it into
  // L2 while the predecessor finishes (the loads themselves follow the wait)
  if (threadIdx.x == 0) prefetch_l2_span(state_in + (int64_t)blockIdx.x * Dv * 2 * D, (size_t)Dv * 2 * D * 4);
  pdl_wait();
  pdl_trigger();
  const int bh = blockIdx.x, b = bh / H, h = bh % H;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int npair = D >> 1, p = lane;
  const bool active = p < npair;
  // the state rows and values first (the long loads), then phases and gate
  const int64_t base = (int64_t)bh * Dv * 2 * D;
  float4 m[RPW];
  float vo[RPW];
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const int o = warp + 8 * r;
    m[r] = make_float4(0.f, 0.f, 0.f, 0.f);
    vo[r] = 0.f;
    if (o < Dv) {
      if (active) m[r] = reinterpret_cast<const float4 *>(state_in + base + (int64_t)o * 2 * D)[p];
      vo[r] = load_any(v, in_dt, b * s_v.b + h * s_v.h + o);
    }
  }
  // this lane's two key / query channels (2p, 2p+1)
  float ck0 = 0.f, sk0 = 0.f, ck1 = 0.f, sk1 = 0.f, cq0 = 0.f, sq0 = 0.f, cq1 = 0.f, sq1 = 0.f;
  if (active) {
    sincosf(load_any(tk, in_dt, b * s_tk.b + h * s_tk.h + 2 * p), &sk0, &ck0);
    sincosf(load_any(tk, in_dt, b * s_tk.b + h * s_tk.h + 2 * p + 1), &sk1, &ck1);
    sincosf(load_any(tq, in_dt, b * s_tq.b + h * s_tq.h + 2 * p), &sq0, &cq0);
    sincosf(load_any(tq, in_dt, b * s_tq.b + h * s_tq.h + 2 * p + 1), &sq1, &cq1);
  }
  const float inv_d = 1.0f / (float)D;
  const float bt_raw = gate_mode == DP_GATE_ONE ? 1.f : load_any(beta, beta_dt, b * s_b.b + h * s_b.h);
  float bt = gate_beta(bt_raw, gate_mode);
  // write key: the read key (real beta) or beta k (complex beta, then bt = 1)
  float wc0 = ck0, ws0 = sk0, wc1 = ck1, ws1 = sk1;
  if (CB) {
    float sp, cp;
    sincosf(bt, &sp, &cp);
    const float br = 1.f + cp;
    wc0 = fmaf(br, ck0, -sp * sk0);
    ws0 = fmaf(br, sk0, sp * ck0);
    wc1 = fmaf(br, ck1, -sp * sk1);
    ws1 = fmaf(br, sk1, sp * ck1);
    bt = 1.f;
  }
  float acc[RPW];
#pragma unroll
  for (int r = 0; r < RPW; ++r) acc[r] = m[r].x * ck0 + m[r].y * sk0 + m[r].z * ck1 + m[r].w * sk1;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1)
#pragma unroll
    for (int r = 0; r < RPW; ++r) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], off);
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const float e = bt * (vo[r] - acc[r] * inv_d);
    m[r].x = fmaf(e, wc0, m[r].x);
    m[r].y = fmaf(e, ws0, m[r].y);
    m[r].z = fmaf(e, wc1, m[r].z);
    m[r].w = fmaf(e, ws1, m[r].w);
    const int o = warp + 8 * r;
    if (o < Dv && active) reinterpret_cast<float4 *>(state_out + base + (int64_t)o * 2 * D)[p] = m[r];
    acc[r] = m[r].x * cq0 + m[r].y * sq0 + m[r].z * cq1 + m[r].w * sq1;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1)
#pragma unroll
    for (int r = 0; r < RPW; ++r) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], off);
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      const int o = warp + 8 * r;
      if (o < Dv) out[b * s_out.b + h * s_out.h + o] = acc[r] * inv_d;
    }
  }
}

}  // namespace
}  // namespace dp

namespace dp {
namespace {
int decode_entry(const char *name, int gate_mode, const float *state_in, float *state_out, const void *theta_k,
                 const void *theta_q, const void *v, const void *beta, int in_dtype, int beta_dtype, float *out,
                 int B, int H, int D, int Dv, const int64_t *strides, void *stream) {
  const std::string n(name);
  DP_REQUIRE(B >= 0 && H >= 0 && D >= 1 && Dv >= 1, DP_ERR_INVALID_ARGUMENT, n + ": bad sizes");
  DP_REQUIRE(gate_mode >= DP_GATE_BETA && gate_mode <= DP_GATE_PHI, DP_ERR_INVALID_ARGUMENT,
             n + ": bad gate mode");
  const bool gate_read = gate_mode != DP_GATE_ONE;
  DP_REQUIRE(valid_dtype(in_dtype) && (!gate_read || valid_dtype(beta_dtype)), DP_ERR_INVALID_ARGUMENT,
             n + ": bad dtype code");
  DP_REQUIRE(D <= 4096, DP_ERR_UNSUPPORTED, n + ": D must be <= 4096");
  if (B == 0 || H == 0) return DP_OK;
  DP_REQUIRE(state_in && state_out && theta_k && theta_q && v && (beta || !gate_read) && out && strides,
             DP_ERR_INVALID_ARGUMENT, n + ": null pointer");
  const bool cbeta = gate_mode == DP_GATE_PHI;
  SeqStrides s[5];
  for (int i = 0; i < 5; ++i) s[i] = SeqStrides{strides[2 * i], strides[2 * i + 1], 0};
  const bool vec4 = (D % 2 == 0) && (reinterpret_cast<uintptr_t>(state_in) % 16 == 0) &&
                    (reinterpret_cast<uintptr_t>(state_out) % 16 == 0);
  const size_t smem = (cbeta ? 6 : 4) * (size_t)D * sizeof(float);
  if (vec4 && D <= 64 && Dv <= 128) {
    auto kern = Dv <= 64 ? (cbeta ? decode_rows_kernel<8, true> : decode_rows_kernel<8, false>)
                         : (cbeta ? decode_rows_kernel<16, true> : decode_rows_kernel<16, false>);
    return pdl_status(launch_pdl(kern, dim3(B * H), dim3(kDecThreads), 0, as_stream(stream), state_in, state_out,
                                 theta_k, theta_q, v, beta, in_dtype, beta_dtype, gate_mode, out, H, D, Dv, s[0],
                                 s[1], s[2], s[3], s[4]),
                      "decode_rows_kernel");
  } else {
    auto kern = vec4 ? (cbeta ? decode_kernel<true, true> : decode_kernel<true, false>)
                     : (cbeta ? decode_kernel<false, true> : decode_kernel<false, false>);
    if (smem > 48 * 1024) {
      const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return set_error(DP_ERR_CUDA, n + ": smem attribute: " + cudaGetErrorString(e));
    }
    return pdl_status(launch_pdl(kern, dim3(B * H), dim3(kDecThreads), smem, as_stream(stream), state_in,
                                 state_out, theta_k, theta_q, v, beta, in_dtype, beta_dtype, gate_mode, out, H, D,
                                 Dv, s[0], s[1], s[2], s[3], s[4]),
                      "decode_kernel");
  }
}
}  // namespace
}  // namespace dp

extern "C" int dp_core_decode(const float *state_in, float *state_out, const void *theta_k,
                              const void *theta_q, const void *v, const void *beta, int in_dtype,
                              int beta_dtype, float *out, int B, int H, int D, int Dv,
                              const int64_t *strides, void *stream) {
  return dp::decode_entry("dp_core_decode", DP_GATE_BETA, state_in, state_out, theta_k, theta_q, v, beta, in_dtype,
                          beta_dtype, out, B, H, D, Dv, strides, stream);
}

extern "C" int dp_core_cbeta_decode(const float *state_in, float *state_out, const void *theta_k,
                                    const void *theta_q, const void *v, const void *phi, int in_dtype,
                                    int phi_dtype, float *out, int B, int H, int D, int Dv,
                                    const int64_t *strides, void *stream) {
  return dp::decode_entry("dp_core_cbeta_decode", DP_GATE_PHI, state_in, state_out, theta_k, theta_q, v, phi, in_dtype,
                          phi_dtype, out, B, H, D, Dv, strides, stream);
}

extern "C" int dp_core_decode_gated(const float *state_in, float *state_out, const void *theta_k,
                                    const void *theta_q, const void *v, const void *gate, int in_dtype,
                                    int gate_dtype, int gate_mode, float *out, int B, int H, int D, int Dv,
                                    const int64_t *strides, void *stream) {
  return dp::decode_entry("dp_core_decode_gated", gate_mode, state_in, state_out, theta_k, theta_q, v, gate,
                          in_dtype, gate_dtype, out, B, H, D, Dv, strides, stream);
}
