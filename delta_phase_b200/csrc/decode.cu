// Single-token decode step of the complex delta rule (memory-bound state update).
//
// Reference: DeltaPhaseHolographicBlock.step (delta_phase/layers.py:279-285):
//   v_old = Re(M conj(k)) / D;  M <- M + beta (v - v_old) k^T;  out = Re(M conj(q)) / D
// (the readout uses the updated state).  Same contract as the never-launched
// _triton_streaming_step_kernel (delta_phase/kernels/triton_chunk_delta.py:125-185),
// but on the interleaved complex64 state, so torch's complex tensor is used as is.
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

// kq: smem (4 x D): cos k, sin k, cos q, sin q.
template <bool kVec4>
__global__ void __launch_bounds__(kDecThreads)
decode_kernel(const float *state_in, float *state_out, const void *__restrict__ tk,
              const void *__restrict__ tq, const void *__restrict__ v,
              const void *__restrict__ beta, int in_dt, int beta_dt, float *__restrict__ out,
              int H, int D, int Dv, SeqStrides s_tk, SeqStrides s_tq, SeqStrides s_v,
              SeqStrides s_b, SeqStrides s_out) {
  extern __shared__ float kq[];
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
  __syncthreads();
  const float inv_d = 1.0f / (float)D;
  const float bt = load_any(beta, beta_dt, b * s_b.b + h * s_b.h);
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
          t.x = fmaf(e, kq[2 * p], t.x);
          t.y = fmaf(e, kq[D + 2 * p], t.y);
          t.z = fmaf(e, kq[2 * p + 1], t.z);
          t.w = fmaf(e, kq[D + 2 * p + 1], t.w);
          reinterpret_cast<float4 *>(row_out)[p] = t;
          r += t.x * kq[2 * D + 2 * p] + t.y * kq[3 * D + 2 * p] + t.z * kq[2 * D + 2 * p + 1] +
               t.w * kq[3 * D + 2 * p + 1];
        }
      }
      for (int p = lane + 128; p < npair; p += 32) {
        float4 t = reinterpret_cast<const float4 *>(row_in)[p];
        t.x = fmaf(e, kq[2 * p], t.x);
        t.y = fmaf(e, kq[D + 2 * p], t.y);
        t.z = fmaf(e, kq[2 * p + 1], t.z);
        t.w = fmaf(e, kq[D + 2 * p + 1], t.w);
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
        m.x = fmaf(e, kq[c], m.x);
        m.y = fmaf(e, kq[D + c], m.y);
        reinterpret_cast<float2 *>(row_out)[c] = m;
        r += m.x * kq[2 * D + c] + m.y * kq[3 * D + c];
      }
      r = warp_sum(r);
      if (lane == 0) out[b * s_out.b + h * s_out.h + o] = r * inv_d;
    }
  }
}

}  // namespace
}  // namespace dp

extern "C" int dp_core_decode(const float *state_in, float *state_out, const void *theta_k,
                              const void *theta_q, const void *v, const void *beta, int in_dtype,
                              int beta_dtype, float *out, int B, int H, int D, int Dv,
                              const int64_t *strides, void *stream) {
  using namespace dp;
  DP_REQUIRE(B >= 0 && H >= 0 && D >= 1 && Dv >= 1, DP_ERR_INVALID_ARGUMENT,
             "dp_core_decode: bad sizes");
  DP_REQUIRE(valid_dtype(in_dtype) && valid_dtype(beta_dtype), DP_ERR_INVALID_ARGUMENT,
             "dp_core_decode: bad dtype code");
  DP_REQUIRE(D <= 4096, DP_ERR_UNSUPPORTED, "dp_core_decode: D must be <= 4096");
  if (B == 0 || H == 0) return DP_OK;
  DP_REQUIRE(state_in && state_out && theta_k && theta_q && v && beta && out && strides,
             DP_ERR_INVALID_ARGUMENT, "dp_core_decode: null pointer");
  SeqStrides s[5];
  for (int i = 0; i < 5; ++i) s[i] = SeqStrides{strides[2 * i], strides[2 * i + 1], 0};
  const bool vec4 = (D % 2 == 0) && (reinterpret_cast<uintptr_t>(state_in) % 16 == 0) &&
                    (reinterpret_cast<uintptr_t>(state_out) % 16 == 0);
  const size_t smem = 4 * (size_t)D * sizeof(float);
  if (vec4)
    decode_kernel<true><<<B * H, kDecThreads, smem, as_stream(stream)>>>(
        state_in, state_out, theta_k, theta_q, v, beta, in_dtype, beta_dtype, out, H, D, Dv, s[0],
        s[1], s[2], s[3], s[4]);
  else
    decode_kernel<false><<<B * H, kDecThreads, smem, as_stream(stream)>>>(
        state_in, state_out, theta_k, theta_q, v, beta, in_dtype, beta_dtype, out, H, D, Dv, s[0],
        s[1], s[2], s[3], s[4]);
  return check_launch("decode_kernel");
}
