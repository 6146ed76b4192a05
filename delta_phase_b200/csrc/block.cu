// Fused glue of DeltaPhaseHolographicBlock.forward (delta_phase/layers.py:177-244):
//   dp_ln_conv_silu : conv_x = n + SiLU(causal_depthwise_conv(n)),  n = LayerNorm(x)
//                     (norm1 and ShortCausalConv1D.forward, layers.py:60-88,178)
//   dp_ln_conv_step : the same for one decode token, with the conv's last k-1 inputs
//                     kept in a (B, d, k-1) state (ShortCausalConv1D.step, layers.py:43-50)
//   dp_layernorm    : s = x (+ residual);  y = LayerNorm(s)  (norm_retrieved, norm2)
// Each is one pass over the (tokens, d) activations instead of the separate
// LayerNorm / transpose / conv / SiLU / add / cast kernels of the module, and each writes
// its output directly in the dtype of the GEMM that consumes it.  LayerNorm statistics
// are two-pass in fp32 (mean, then the mean of squared deviations), like torch's.
#include <string>

#include "dp_common.cuh"

namespace dp {
namespace {

constexpr int kBlkThreads = 256;

template <typename T>
__device__ __forceinline__ void store_f32_as(T *p, float v);
template <>
__device__ __forceinline__ void store_f32_as<float>(float *p, float v) { *p = v; }
template <>
__device__ __forceinline__ void store_f32_as<__nv_bfloat16>(__nv_bfloat16 *p, float v) { *p = __float2bfloat16_rn(v); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
  return v;
}

// Grid (ceil(L / T), B); rows t0 - (k - 1) .. t0 + T - 1 of batch b are normalised into
// shared memory (zeros before the sequence start: the conv's zero padding), then thread
// c walks column c through the T tokens of the tile.
template <typename InT, typename OutT>
__global__ void __launch_bounds__(kBlkThreads)
ln_conv_silu_kernel(const InT *__restrict__ x, const float *__restrict__ ln_w, const float *__restrict__ ln_b,
                    float eps, const float *__restrict__ conv_w, const float *__restrict__ conv_b,
                    OutT *__restrict__ out, int L, int d, int k, int T) {
  extern __shared__ float nrm[];  // (T + k - 1) x d
  const int b = blockIdx.y, t0 = blockIdx.x * T;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = kBlkThreads / 32;
  const int rows = T + k - 1;
  const float inv_d = 1.0f / (float)d;
  for (int r = warp; r < rows; r += nwarps) {
    const int t = t0 - (k - 1) + r;
    float *nr = nrm + (size_t)r * d;
    if (t < 0 || t >= L) {
      for (int c = lane; c < d; c += 32) nr[c] = 0.f;
      continue;
    }
    const InT *xr = x + ((size_t)b * L + t) * d;
    float s = 0.f;
    for (int c = lane; c < d; c += 32) {
      const float v = to_f32(xr[c]);
      nr[c] = v;
      s += v;
    }
    const float mean = warp_sum(s) * inv_d;
    float q = 0.f;
    for (int c = lane; c < d; c += 32) {
      const float dv = nr[c] - mean;
      q = fmaf(dv, dv, q);
    }
    const float rstd = rsqrtf(warp_sum(q) * inv_d + eps);
    for (int c = lane; c < d; c += 32) nr[c] = fmaf((nr[c] - mean) * rstd, ln_w[c], ln_b[c]);
  }
  __syncthreads();
  for (int c = threadIdx.x; c < d; c += kBlkThreads) {
    float w[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) w[j] = j < k ? conv_w[(size_t)c * k + j] : 0.f;
    const float cb = conv_b ? conv_b[c] : 0.f;
    for (int i = 0; i < T && t0 + i < L; ++i) {
      float acc = cb;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j < k) acc = fmaf(w[j], nrm[(size_t)(i + j) * d + c], acc);
      const float silu = acc / (1.f + __expf(-acc));
      store_f32_as(out + ((size_t)b * L + t0 + i) * d + c, nrm[(size_t)(i + k - 1) * d + c] + silu);
    }
  }
}

// One warp per row: s = x (+ res); y = LayerNorm(s); the row stays in L1 between passes.
template <typename InT, typename OutT>
__global__ void __launch_bounds__(kBlkThreads)
layernorm_kernel(const InT *x, const float *res, const float *__restrict__ ln_w,
                 const float *__restrict__ ln_b, float eps, float *__restrict__ sum_out, OutT *__restrict__ y,
                 int64_t rows, int d) {
  pdl_wait();
  pdl_trigger();
  const int64_t r = (int64_t)blockIdx.x * (kBlkThreads / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const InT *xr = x + r * d;
  const float *rr = res ? res + r * d : nullptr;
  const float inv_d = 1.0f / (float)d;
  float s = 0.f;
  for (int c = lane; c < d; c += 32) {
    float v = to_f32(xr[c]);
    if (rr) v += rr[c];
    if (sum_out) sum_out[r * d + c] = v;
    s += v;
  }
  const float mean = warp_sum(s) * inv_d;
  float q = 0.f;
  for (int c = lane; c < d; c += 32) {
    float v = to_f32(xr[c]);
    if (rr) v += rr[c];
    const float dv = v - mean;
    q = fmaf(dv, dv, q);
  }
  const float rstd = rsqrtf(warp_sum(q) * inv_d + eps);
  for (int c = lane; c < d; c += 32) {
    float v = to_f32(xr[c]);
    if (rr) v += rr[c];
    store_f32_as(y + r * d + c, fmaf((v - mean) * rstd, ln_w[c], ln_b[c]));
  }
}

// Eight consecutive values <-> float: 16-byte (bf16) or two 16-byte (float) accesses.
__device__ __forceinline__ void load8(const float *p, float (&v)[8]) {
  const float4 a = reinterpret_cast<const float4 *>(p)[0], b = reinterpret_cast<const float4 *>(p)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void load8(const __nv_bfloat16 *p, float (&v)[8]) {
  const uint4 a = *reinterpret_cast<const uint4 *>(p);
  const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w[i]));
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void store8(float *p, const float (&v)[8]) {
  reinterpret_cast<float4 *>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4 *>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}
__device__ __forceinline__ void store8(__nv_bfloat16 *p, const float (&v)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t *>(&h);
  }
  *reinterpret_cast<uint4 *>(p) = make_uint4(w[0], w[1], w[2], w[3]);
}

// The same LayerNorm with the row held in registers: one warp per row, lane l holds the
// eight-value groups l, l + 32, ... (NG groups, d = 256 NG), every global access 16 bytes
// wide and issued before the reductions.  The row is read once, not three times, and at
// the few rows of a decode step the load latency is paid once per row.
template <typename InT, typename OutT, int NG>
__global__ void __launch_bounds__(128)
layernorm_reg_kernel(const InT *x, const float *res, const float *__restrict__ ln_w,
                     const float *__restrict__ ln_b, float eps, float *__restrict__ sum_out, OutT *__restrict__ y,
                     int64_t rows) {
  constexpr int d = 256 * NG;
  pdl_wait();
  pdl_trigger();
  const int64_t r = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  float v[NG][8];
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    const int c0 = 8 * (lane + 32 * g);
    load8(x + r * d + c0, v[g]);
    if (res) {
      float rv[8];
      load8(res + r * d + c0, rv);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[g][i] += rv[i];
    }
  }
  float s = 0.f;
#pragma unroll
  for (int g = 0; g < NG; ++g)
#pragma unroll
    for (int i = 0; i < 8; ++i) s += v[g][i];
  const float mean = warp_sum(s) * (1.0f / d);
  float q = 0.f;
#pragma unroll
  for (int g = 0; g < NG; ++g)
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float dv = v[g][i] - mean;
      q = fmaf(dv, dv, q);
    }
  const float rstd = rsqrtf(warp_sum(q) * (1.0f / d) + eps);
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    const int c0 = 8 * (lane + 32 * g);
    if (sum_out) store8(sum_out + r * d + c0, v[g]);
    float w[8], bb[8], o[8];
    load8(ln_w + c0, w);
    load8(ln_b + c0, bb);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = fmaf((v[g][i] - mean) * rstd, w[i], bb[i]);
    store8(y + r * d + c0, o);
  }
}

__device__ __forceinline__ void load4(const float *p, float (&v)[4]) {
  const float4 a = *reinterpret_cast<const float4 *>(p);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
}
__device__ __forceinline__ void load4(const __nv_bfloat16 *p, float (&v)[4]) {
  const uint2 a = *reinterpret_cast<const uint2 *>(p);
  const float2 f0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&a.x));
  const float2 f1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&a.y));
  v[0] = f0.x; v[1] = f0.y; v[2] = f1.x; v[3] = f1.y;
}
__device__ __forceinline__ void store4(float *p, const float (&v)[4]) {
  *reinterpret_cast<float4 *>(p) = make_float4(v[0], v[1], v[2], v[3]);
}
__device__ __forceinline__ void store4(__nv_bfloat16 *p, const float (&v)[4]) {
  __nv_bfloat162 h0 = __floats2bfloat162_rn(v[0], v[1]), h1 = __floats2bfloat162_rn(v[2], v[3]);
  *reinterpret_cast<uint2 *>(p) = make_uint2(*reinterpret_cast<uint32_t *>(&h0), *reinterpret_cast<uint32_t *>(&h1));
}

// The same pass for the usual shapes (conv kernel size 4, d = 256 NG <= 1024, 16-byte
// aligned rows), at HBM speed: a CTA takes 32 tokens of one sequence; first each warp
// computes the LayerNorm statistics of rows t0 - 3 .. t0 + 31 from registers (one
// 16-byte-wide read of the row), then thread t walks channels t + 256 j down the 35 rows,
// normalising on the fly and keeping the three previous normalised values in registers
// for the depthwise conv (four consecutive channels per thread, 16-byte loads).  Shared
// memory holds only the 2 x 35 statistics (the kernel
// above stages the normalised rows, 77 KB, and runs at a fraction of the bandwidth).
constexpr int kConvRowsT = 32;

template <typename InT, typename OutT, int NG>
__global__ void __launch_bounds__(kBlkThreads)
ln_conv_silu_rows_kernel(const InT *x, const float *__restrict__ ln_w, const float *__restrict__ ln_b, float eps,
                         const float *__restrict__ conv_w, const float *__restrict__ conv_b,
                         OutT *__restrict__ out, int L) {
  constexpr int d = 256 * NG, K = 4, R = kConvRowsT + K - 1;
  __shared__ float s_mean[R], s_rstd[R];
  const int b = blockIdx.y, t0 = blockIdx.x * kConvRowsT;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int r = warp; r < R; r += kBlkThreads / 32) {
    const int t = t0 - (K - 1) + r;
    if (t < 0 || t >= L) {  // the conv's zero padding (t < 0); rows past L are not used
      if (lane == 0) s_mean[r] = s_rstd[r] = 0.f;
      continue;
    }
    const InT *xr = x + ((size_t)b * L + t) * d;
    float v[NG][8];
#pragma unroll
    for (int g = 0; g < NG; ++g) load8(xr + 8 * (lane + 32 * g), v[g]);
    float s = 0.f;
#pragma unroll
    for (int g = 0; g < NG; ++g)
#pragma unroll
      for (int i = 0; i < 8; ++i) s += v[g][i];
    const float mean = warp_sum(s) * (1.0f / d);
    float q = 0.f;
#pragma unroll
    for (int g = 0; g < NG; ++g)
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float dv = v[g][i] - mean;
        q = fmaf(dv, dv, q);
      }
    const float rstd = rsqrtf(warp_sum(q) * (1.0f / d) + eps);
    if (lane == 0) {
      s_mean[r] = mean;
      s_rstd[r] = rstd;
    }
  }
  __syncthreads();
  // four consecutive channels per thread: 16-byte loads of x and the parameters
#pragma unroll 1
  for (int g = threadIdx.x; g < d / 4; g += kBlkThreads) {
    const int c = 4 * g;
    float4 w[4];  // taps of channels c .. c + 3
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = reinterpret_cast<const float4 *>(conv_w)[c + i];
    const float4 lw = *reinterpret_cast<const float4 *>(ln_w + c), lb = *reinterpret_cast<const float4 *>(ln_b + c);
    const float4 cb = conv_b ? *reinterpret_cast<const float4 *>(conv_b + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    const float lwv[4] = {lw.x, lw.y, lw.z, lw.w}, lbv[4] = {lb.x, lb.y, lb.z, lb.w};
    const float cbv[4] = {cb.x, cb.y, cb.z, cb.w};
    float n0[4] = {0.f, 0.f, 0.f, 0.f}, n1[4] = {0.f, 0.f, 0.f, 0.f}, n2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
    for (int r = 0; r < R; ++r) {
      const int t = t0 - (K - 1) + r;
      float n[4] = {0.f, 0.f, 0.f, 0.f};
      if (t >= 0 && t < L) {
        float xv[4];
        load4(x + ((size_t)b * L + t) * d + c, xv);
        const float mu = s_mean[r], rs = s_rstd[r];
#pragma unroll
        for (int i = 0; i < 4; ++i) n[i] = fmaf((xv[i] - mu) * rs, lwv[i], lbv[i]);
      }
      if (r >= K - 1 && t < L) {
        float o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float acc = fmaf(w[i].x, n0[i], cbv[i]);
          acc = fmaf(w[i].y, n1[i], acc);
          acc = fmaf(w[i].z, n2[i], acc);
          acc = fmaf(w[i].w, n[i], acc);
          o[i] = n[i] + acc / (1.f + __expf(-acc));
        }
        store4(out + ((size_t)b * L + t) * d + c, o);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        n0[i] = n1[i];
        n1[i] = n2[i];
        n2[i] = n[i];
      }
    }
  }
}

// Decode step of norm1 + ShortCausalConv1D.step (layers.py:43-50,182-190): one CTA per
// sequence.  n = LayerNorm(x_t); out = n + SiLU(b + sum_{j<k-1} w[j] state[j] + w[k-1] n);
// state (d, k-1) float32 shifts left and takes n (the conv's last k-1 inputs).
template <typename InT, typename OutT>
__global__ void __launch_bounds__(kBlkThreads)
ln_conv_step_kernel(const InT *x, const float *__restrict__ ln_w, const float *__restrict__ ln_b,
                    float eps, const float *__restrict__ conv_w, const float *__restrict__ conv_b,
                    float *__restrict__ state, OutT *__restrict__ out, int d, int k) {
  __shared__ float red[kBlkThreads / 32];
  __shared__ float stat[2];
  if (threadIdx.x == 0 && k > 1)  // this row's conv state, into L2 before the wait
    prefetch_l2_span(state + (size_t)blockIdx.x * d * (k - 1), (size_t)d * (k - 1) * 4);
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const InT *xr = x + (size_t)b * d;
  const float inv_d = 1.0f / (float)d;
  float s = 0.f;
  for (int c = tid; c < d; c += kBlkThreads) s += to_f32(xr[c]);
  s = warp_sum(s);
  if (lane == 0) red[warp] = s;
  __syncthreads();
  if (tid == 0) {
    float t = 0.f;
    for (int w = 0; w < kBlkThreads / 32; ++w) t += red[w];
    stat[0] = t * inv_d;
  }
  __syncthreads();
  const float mean = stat[0];
  float q = 0.f;
  for (int c = tid; c < d; c += kBlkThreads) {
    const float dv = to_f32(xr[c]) - mean;
    q = fmaf(dv, dv, q);
  }
  q = warp_sum(q);
  if (lane == 0) red[warp] = q;
  __syncthreads();
  if (tid == 0) {
    float t = 0.f;
    for (int w = 0; w < kBlkThreads / 32; ++w) t += red[w];
    stat[1] = rsqrtf(t * inv_d + eps);
  }
  __syncthreads();
  const float rstd = stat[1];
  for (int c = tid; c < d; c += kBlkThreads) {
    const float n = fmaf((to_f32(xr[c]) - mean) * rstd, ln_w[c], ln_b[c]);
    float *st = state + ((size_t)b * d + c) * (k - 1);
    const float *w = conv_w + (size_t)c * k;
    float acc = conv_b ? conv_b[c] : 0.f;
    for (int j = 0; j < k - 1; ++j) acc = fmaf(w[j], st[j], acc);
    acc = fmaf(w[k - 1], n, acc);
    for (int j = 0; j + 1 < k - 1; ++j) st[j] = st[j + 1];
    if (k > 1) st[k - 2] = n;
    store_f32_as(out + (size_t)b * d + c, n + acc / (1.f + __expf(-acc)));
  }
}

// The same step for the usual shapes (conv kernel size 4, d = 256 CPT <= 1024): thread t
// owns channels t + 256 j; every load of the row -- x, the LayerNorm and conv parameters,
// the three state values -- is issued right after the wait, before the two reductions,
// so the step pays one memory round trip instead of three.
template <typename InT, typename OutT, int CPT>
__global__ void __launch_bounds__(kBlkThreads)
ln_conv_step_reg_kernel(const InT *x, const float *__restrict__ ln_w, const float *__restrict__ ln_b, float eps,
                        const float *__restrict__ conv_w, const float *__restrict__ conv_b, float *state,
                        OutT *__restrict__ out) {
  constexpr int d = kBlkThreads * CPT;
  __shared__ float red[2][kBlkThreads / 32];
  const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float *st = state + (size_t)b * d * 3;
  if (tid == 0) prefetch_l2_span(st, (size_t)d * 3 * 4);  // before the wait: see the kernel above
  pdl_wait();
  pdl_trigger();
  float xv[CPT], w[CPT], bb[CPT], cb[CPT], s0[CPT], s1[CPT], s2[CPT];
  float4 cw[CPT];
#pragma unroll
  for (int j = 0; j < CPT; ++j) {
    const int c = tid + kBlkThreads * j;
    xv[j] = to_f32(x[(size_t)b * d + c]);
    w[j] = ln_w[c];
    bb[j] = ln_b[c];
    cb[j] = conv_b ? conv_b[c] : 0.f;
    cw[j] = reinterpret_cast<const float4 *>(conv_w)[c];  // w[c][0..3], 16-byte aligned rows
    s0[j] = st[c * 3];
    s1[j] = st[c * 3 + 1];
    s2[j] = st[c * 3 + 2];
  }
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < CPT; ++j) s += xv[j];
  s = warp_sum(s);
  if (lane == 0) red[0][warp] = s;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < kBlkThreads / 32; ++i) t += red[0][i];
  const float mean = t * (1.0f / d);
  float q = 0.f;
#pragma unroll
  for (int j = 0; j < CPT; ++j) {
    const float dv = xv[j] - mean;
    q = fmaf(dv, dv, q);
  }
  q = warp_sum(q);
  if (lane == 0) red[1][warp] = q;
  __syncthreads();
  t = 0.f;
#pragma unroll
  for (int i = 0; i < kBlkThreads / 32; ++i) t += red[1][i];
  const float rstd = rsqrtf(t * (1.0f / d) + eps);
#pragma unroll
  for (int j = 0; j < CPT; ++j) {
    const int c = tid + kBlkThreads * j;
    const float n = fmaf((xv[j] - mean) * rstd, w[j], bb[j]);
    float acc = cb[j];
    acc = fmaf(cw[j].x, s0[j], acc);
    acc = fmaf(cw[j].y, s1[j], acc);
    acc = fmaf(cw[j].z, s2[j], acc);
    acc = fmaf(cw[j].w, n, acc);
    st[c * 3] = s1[j];
    st[c * 3 + 1] = s2[j];
    st[c * 3 + 2] = n;
    store_f32_as(out + (size_t)b * d + c, n + acc / (1.f + __expf(-acc)));
  }
}

}  // namespace
}  // namespace dp

extern "C" int dp_ln_conv_silu(const void *x, int x_dtype, const float *ln_w, const float *ln_b, float eps,
                               const float *conv_w, const float *conv_b, void *out, int out_dtype, int B, int L,
                               int d, int k, void *stream) {
  using namespace dp;
  DP_REQUIRE(B >= 0 && L >= 0 && d >= 1 && k >= 1, DP_ERR_INVALID_ARGUMENT, "dp_ln_conv_silu: bad sizes");
  DP_REQUIRE(k <= 8, DP_ERR_UNSUPPORTED, "dp_ln_conv_silu: kernel size must be <= 8");
  DP_REQUIRE((x_dtype == DP_F32 || x_dtype == DP_BF16) && (out_dtype == DP_F32 || out_dtype == DP_BF16),
             DP_ERR_INVALID_ARGUMENT, "dp_ln_conv_silu: dtypes must be float32 or bfloat16");
  if (B == 0 || L == 0) return DP_OK;
  DP_REQUIRE(x && ln_w && ln_b && conv_w && out, DP_ERR_INVALID_ARGUMENT, "dp_ln_conv_silu: null pointer");
  cudaStream_t st0 = as_stream(stream);
  auto al16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (k == 4 && d % kBlkThreads == 0 && d <= 4 * kBlkThreads && al16(x) && al16(conv_w) && al16(ln_w) &&
      al16(ln_b) && al16(conv_b) && al16(out) && (L + kConvRowsT - 1) / kConvRowsT < (1 << 30)) {
    const dim3 grid((L + kConvRowsT - 1) / kConvRowsT, B);
    auto launch = [&](auto xt, auto ot) {
      using XT = decltype(xt);
      using OT = decltype(ot);
      auto kern = d == 256 ? ln_conv_silu_rows_kernel<XT, OT, 1>
                  : d == 512 ? ln_conv_silu_rows_kernel<XT, OT, 2>
                  : d == 768 ? ln_conv_silu_rows_kernel<XT, OT, 3>
                             : ln_conv_silu_rows_kernel<XT, OT, 4>;
      kern<<<grid, kBlkThreads, 0, st0>>>(static_cast<const XT *>(x), ln_w, ln_b, eps, conv_w, conv_b,
                                           static_cast<OT *>(out), L);
    };
    if (x_dtype == DP_F32) {
      if (out_dtype == DP_F32) launch(float{}, float{});
      else launch(float{}, __nv_bfloat16{});
    } else {
      if (out_dtype == DP_F32) launch(__nv_bfloat16{}, float{});
      else launch(__nv_bfloat16{}, __nv_bfloat16{});
    }
    return check_launch("ln_conv_silu_rows_kernel");
  }
  int T = 16;
  while (T > 1 && (size_t)(T + k - 1) * d * sizeof(float) > 200 * 1024) T >>= 1;
  const size_t smem = (size_t)(T + k - 1) * d * sizeof(float);
  DP_REQUIRE(smem <= 227 * 1024, DP_ERR_UNSUPPORTED, "dp_ln_conv_silu: d too large");
  dim3 grid((L + T - 1) / T, B);
  cudaStream_t st = as_stream(stream);
  cudaError_t attr_err = cudaSuccess;
  auto launch = [&](auto xt, auto ot) {
    using XT = decltype(xt);
    using OT = decltype(ot);
    attr_err = cudaFuncSetAttribute(ln_conv_silu_kernel<XT, OT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (attr_err != cudaSuccess) return;
    ln_conv_silu_kernel<XT, OT><<<grid, kBlkThreads, smem, st>>>(static_cast<const XT *>(x), ln_w, ln_b, eps,
                                                                 conv_w, conv_b, static_cast<OT *>(out), L, d, k, T);
  };
  if (x_dtype == DP_F32) {
    if (out_dtype == DP_F32) launch(float{}, float{});
    else launch(float{}, __nv_bfloat16{});
  } else {
    if (out_dtype == DP_F32) launch(__nv_bfloat16{}, float{});
    else launch(__nv_bfloat16{}, __nv_bfloat16{});
  }
  if (attr_err != cudaSuccess)
    return set_error(DP_ERR_CUDA, std::string("ln_conv_silu smem attr: ") + cudaGetErrorString(attr_err));
  return check_launch("ln_conv_silu_kernel");
}

extern "C" int dp_layernorm(const void *x, int x_dtype, const float *residual, const float *ln_w,
                            const float *ln_b, float eps, float *sum_out, void *y, int y_dtype, int64_t rows, int d,
                            void *stream) {
  using namespace dp;
  DP_REQUIRE(rows >= 0 && d >= 1, DP_ERR_INVALID_ARGUMENT, "dp_layernorm: bad sizes");
  DP_REQUIRE((x_dtype == DP_F32 || x_dtype == DP_BF16) && (y_dtype == DP_F32 || y_dtype == DP_BF16),
             DP_ERR_INVALID_ARGUMENT, "dp_layernorm: dtypes must be float32 or bfloat16");
  if (rows == 0) return DP_OK;
  DP_REQUIRE(x && ln_w && ln_b && y, DP_ERR_INVALID_ARGUMENT, "dp_layernorm: null pointer");
  const int64_t blocks = (rows + kBlkThreads / 32 - 1) / (kBlkThreads / 32);
  DP_REQUIRE(blocks < (1ll << 31), DP_ERR_UNSUPPORTED, "dp_layernorm: too many rows");
  cudaStream_t st = as_stream(stream);
  auto al16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (d % 256 == 0 && d <= 1024 && al16(x) && al16(residual) && al16(ln_w) && al16(ln_b) && al16(sum_out) &&
      al16(y) && (rows + 3) / 4 < (1ll << 31)) {
    // row in registers (d = 256, 512, 768, 1024), four rows per CTA
    const unsigned rb = (unsigned)((rows + 3) / 4);
    auto launch_reg = [&](auto xt, auto ot) {
      using XT = decltype(xt);
      using OT = decltype(ot);
      const XT *xp = static_cast<const XT *>(x);
      OT *yp = static_cast<OT *>(y);
      auto kern = d == 256 ? layernorm_reg_kernel<XT, OT, 1>
                  : d == 512 ? layernorm_reg_kernel<XT, OT, 2>
                  : d == 768 ? layernorm_reg_kernel<XT, OT, 3>
                             : layernorm_reg_kernel<XT, OT, 4>;
      return launch_pdl(kern, dim3(rb), dim3(128), 0, st, xp, residual, ln_w, ln_b, eps, sum_out, yp, rows);
    };
    cudaError_t e;
    if (x_dtype == DP_F32)
      e = y_dtype == DP_F32 ? launch_reg(float{}, float{}) : launch_reg(float{}, __nv_bfloat16{});
    else
      e = y_dtype == DP_F32 ? launch_reg(__nv_bfloat16{}, float{}) : launch_reg(__nv_bfloat16{}, __nv_bfloat16{});
    return pdl_status(e, "layernorm_reg_kernel");
  }
  auto launch = [&](auto xt, auto ot) {
    using XT = decltype(xt);
    using OT = decltype(ot);
    return launch_pdl(layernorm_kernel<XT, OT>, dim3((unsigned)blocks), dim3(kBlkThreads), 0, st,
                      static_cast<const XT *>(x), residual, ln_w, ln_b, eps, sum_out, static_cast<OT *>(y), rows, d);
  };
  cudaError_t e;
  if (x_dtype == DP_F32)
    e = y_dtype == DP_F32 ? launch(float{}, float{}) : launch(float{}, __nv_bfloat16{});
  else
    e = y_dtype == DP_F32 ? launch(__nv_bfloat16{}, float{}) : launch(__nv_bfloat16{}, __nv_bfloat16{});
  return pdl_status(e, "layernorm_kernel");
}

extern "C" int dp_ln_conv_step(const void *x, int x_dtype, const float *ln_w, const float *ln_b, float eps,
                               const float *conv_w, const float *conv_b, float *conv_state, void *out,
                               int out_dtype, int B, int d, int k, void *stream) {
  using namespace dp;
  DP_REQUIRE(B >= 0 && d >= 1 && k >= 1, DP_ERR_INVALID_ARGUMENT, "dp_ln_conv_step: bad sizes");
  DP_REQUIRE((x_dtype == DP_F32 || x_dtype == DP_BF16) && (out_dtype == DP_F32 || out_dtype == DP_BF16),
             DP_ERR_INVALID_ARGUMENT, "dp_ln_conv_step: dtypes must be float32 or bfloat16");
  if (B == 0) return DP_OK;
  DP_REQUIRE(x && ln_w && ln_b && conv_w && out && (k == 1 || conv_state), DP_ERR_INVALID_ARGUMENT,
             "dp_ln_conv_step: null pointer");
  cudaStream_t st = as_stream(stream);
  const bool reg = k == 4 && d % kBlkThreads == 0 && d <= 4 * kBlkThreads &&
                   (reinterpret_cast<uintptr_t>(conv_w) & 15) == 0;
  auto launch = [&](auto xt, auto ot) {
    using XT = decltype(xt);
    using OT = decltype(ot);
    if (reg) {
      auto kern = d == 256 ? ln_conv_step_reg_kernel<XT, OT, 1>
                  : d == 512 ? ln_conv_step_reg_kernel<XT, OT, 2>
                  : d == 768 ? ln_conv_step_reg_kernel<XT, OT, 3>
                             : ln_conv_step_reg_kernel<XT, OT, 4>;
      return launch_pdl(kern, dim3(B), dim3(kBlkThreads), 0, st, static_cast<const XT *>(x), ln_w, ln_b, eps,
                        conv_w, conv_b, conv_state, static_cast<OT *>(out));
    }
    return launch_pdl(ln_conv_step_kernel<XT, OT>, dim3(B), dim3(kBlkThreads), 0, st, static_cast<const XT *>(x),
                      ln_w, ln_b, eps, conv_w, conv_b, conv_state, static_cast<OT *>(out), d, k);
  };
  cudaError_t e;
  if (x_dtype == DP_F32)
    e = out_dtype == DP_F32 ? launch(float{}, float{}) : launch(float{}, __nv_bfloat16{});
  else
    e = out_dtype == DP_F32 ? launch(__nv_bfloat16{}, float{}) : launch(__nv_bfloat16{}, __nv_bfloat16{});
  return pdl_status(e, "ln_conv_step_kernel");
}
