// Spectral Lerp FFN: parameter fold and forward.
//
// Reference: LearnableSubstrateLerpFFN.forward (delta_phase/layers.py:119-141) and the
// bases of delta_phase/spectral.py:4-35, mcarbonell/delta-phase v1.3.0.
//
// Per branch b (FWHT, DCT-II, Haar) the reference computes h = M_b x, the multi-bank
// activation a[k, i] = cos(h_i + phi1[k, i]) w1[k, i] + sin(h_i + phi2[k, i]) w2[k, i],
// c = W_c a (shared combine) and M_b^T c, then mixes the branches with softmax router
// weights.  By angle addition a[k, i] = alpha[k, i] cos h_i + gamma[k, i] sin h_i with
//   alpha = w1 cos phi1 + w2 sin phi2,   gamma = w2 cos phi2 - w1 sin phi1,
// so the whole FFN is linear in z = [cos h_b, sin h_b]_b (6d values per token):
//   y = z F,  F[(2b+s) d + i, j] = w_b sum_m (sum_k coef_{b,s}[k, i] W_c[m, k d + i]) M_b[m, j].
// dp_ffn_fold builds F once per parameter update (float64 accumulation); the forward
// then needs 6d sincos and one (tokens x 6d) x (6d x d) GEMM per call -- half the
// multiply-adds of the reference's three (tokens x nb d) x (nb d x d) combines at nb = 4,
// and none of its six dense d x d transform GEMMs except the DCT.
#include <array>
#include <mutex>
#include <string>
#include <type_traits>

#include "dp_common.cuh"

namespace dp {

bool gemm_tc_supported(int es, const void *A, const void *B, int M, int N, int K, int64_t lda, int64_t ldb,
                       int bn_max = 256);
int gemm_tc(int es, const void *A, int64_t lda, const void *B, int64_t ldb, void *C, int64_t ldc, int M, int N, int K,
            int epi, cudaStream_t stream, int64_t sin_off = 0, int bn_max = 256);

namespace {

// ---------------------------------------------------------------- fold
constexpr int kFoldTile = 32;
// token counts up to which dp_ffn_fwd computes the three feature branches of a token on
// three warps (decode batches) instead of one
constexpr int kFeatSplitTokens = 512;

// grid (d/32, d/32, 6): z = 2*branch + s.  One thread per output, float64 accumulation.
__global__ void __launch_bounds__(kFoldTile * 8)
ffn_fold_kernel(const float *__restrict__ logits, const float *__restrict__ mats,
                const float *__restrict__ banks, const float *__restrict__ combine,
                float *__restrict__ F, int d, int nb) {
  __shared__ double At[kFoldTile][kFoldTile + 1];  // Wt[m][i] tile (m along rows)
  __shared__ double Bt[kFoldTile][kFoldTile + 1];  // M_b[m][j] tile
  const int br = blockIdx.z >> 1, sc = blockIdx.z & 1;
  const int i0 = blockIdx.y * kFoldTile, j0 = blockIdx.x * kFoldTile;
  const int tx = threadIdx.x % kFoldTile, ty = threadIdx.x / kFoldTile;  // ty in [0, 8)
  // router weight w_b = softmax(logits)_b
  double lmax = fmax(fmax((double)logits[0], (double)logits[1]), (double)logits[2]);
  double den = exp(logits[0] - lmax) + exp(logits[1] - lmax) + exp(logits[2] - lmax);
  const double wb = exp(logits[br] - lmax) / den;
  const float *Mb = mats + (size_t)br * d * d;
  const float *phi1 = banks + ((size_t)br * 4 + 0) * nb * d;
  const float *phi2 = banks + ((size_t)br * 4 + 1) * nb * d;
  const float *w1 = banks + ((size_t)br * 4 + 2) * nb * d;
  const float *w2 = banks + ((size_t)br * 4 + 3) * nb * d;
  double acc[4] = {0, 0, 0, 0};
  for (int m0 = 0; m0 < d; m0 += kFoldTile) {
    for (int r = ty; r < kFoldTile; r += 8) {
      const int m = m0 + r, i = i0 + tx;
      double wt = 0.0, mv = 0.0;
      if (m < d && i < d)
      for (int k = 0; k < nb; ++k) {
        const size_t ki = (size_t)k * d + i;
        const double p1 = phi1[ki], p2 = phi2[ki], a1 = w1[ki], a2 = w2[ki];
        const double coef = sc == 0 ? a1 * cos(p1) + a2 * sin(p2) : a2 * cos(p2) - a1 * sin(p1);
        wt += coef * (double)combine[(size_t)m * nb * d + ki];
      }
      if (m < d && j0 + tx < d) mv = (double)Mb[(size_t)m * d + j0 + tx];
      At[r][tx] = wt;
      Bt[r][tx] = mv;
    }
    __syncthreads();
#pragma unroll 8
    for (int mm = 0; mm < kFoldTile; ++mm) {
      const double bj = Bt[mm][tx];
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[q] += At[mm][ty + 8 * q] * bj;
    }
    __syncthreads();
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int i = i0 + ty + 8 * q, j = j0 + tx;
    if (i < d && j < d) F[((size_t)blockIdx.z * d + i) * d + j] = (float)(wb * acc[q]);
  }
}

// ---------------------------------------------------------------- transforms
// One CTA per token row; four d-float shared buffers; writes the 6d-value row of z.
template <typename T>
__global__ void __launch_bounds__(256)
ffn_features_kernel(const T *__restrict__ x, const float *__restrict__ hdct, T *__restrict__ z, int d,
                    int log2d) {
  extern __shared__ float sm[];
  float *a = sm;       // FWHT work vector
  float *hb = a + d;   // Haar work vector
  float *ho = hb + d;  // Haar output
  float *tmp = ho + d; // Haar ping-pong buffer
  const int tid = threadIdx.x, nt = blockDim.x;
  const int64_t row = blockIdx.x;
  const T *xr = x + row * d;
  for (int i = tid; i < d; i += nt) {
    const float xv = to_f32(xr[i]);
    a[i] = xv;
    hb[i] = xv;
  }
  __syncthreads();
  // Sylvester FWHT in natural order: (H x)[i] = sum_j (-1)^{popcount(i & j)} x[j]
  for (int len = 1; len < d; len <<= 1) {
    for (int p = tid; p < d / 2; p += nt) {
      const int i = (p / len) * 2 * len + (p % len);
      const float u = a[i], w = a[i + len];
      a[i] = u + w;
      a[i + len] = u - w;
    }
    __syncthreads();
  }
  // the reference's recursive Haar: high[i] = (x[2i] - x[2i+1]) / sqrt2 on the
  // current level, low = (x[:n/2] + x[n/2:]) / sqrt2 recursed (spectral.py:25-35)
  const float r2 = 0.70710678118654752f;
  float *src = hb, *dst = tmp;
  for (int n = d; n > 1; n >>= 1) {
    const int half = n >> 1;
    for (int i = tid; i < half; i += nt) {
      ho[half + i] = (src[2 * i] - src[2 * i + 1]) * r2;
      dst[i] = (src[i] + src[i + half]) * r2;
    }
    __syncthreads();
    float *t = src;
    src = dst;
    dst = t;
  }
  if (tid == 0) ho[0] = src[0];
  __syncthreads();
  const float inv_sqrt_d = rsqrtf((float)d);
  T *zr = z + row * 6 * d;
  const float *hd = hdct ? hdct + row * d : nullptr;
  for (int i = tid; i < d; i += nt) {
    float s, c;
    sincosf(a[i] * inv_sqrt_d, &s, &c);
    zr[i] = from_f32<T>(c);
    zr[d + i] = from_f32<T>(s);
    if (hd) {
      sincosf(hd[i], &s, &c);
      zr[2 * d + i] = from_f32<T>(c);
      zr[3 * d + i] = from_f32<T>(s);
    }
    sincosf(ho[i], &s, &c);
    zr[4 * d + i] = from_f32<T>(c);
    zr[5 * d + i] = from_f32<T>(s);
  }
}

// Warp-per-token features for d = 32 R (256, 512, 1024): the token row lives in registers, lane l
// holding x[R l .. R l + R).  FWHT butterflies on bits below log2 R run inside a lane,
// the five higher bits across lanes with shuffles; the reference's recursive Haar takes
// adjacent-pair differences inside a lane and folds the upper half of the current level
// onto the lower half with a shuffle down, until one lane holds the last R values.
// No shared memory and no block barriers; sin / cos through sincos_2pi_fast.
template <typename T>
__device__ __forceinline__ void store_pair(T *p, float a, float b) {
  if constexpr (sizeof(T) == 2) {
    *reinterpret_cast<uint32_t *>(p) = pack_bf16_rne(a, b);
  } else {
    *reinterpret_cast<float2 *>(p) = make_float2(a, b);
  }
}

// cos and sin of n consecutive values (n even, p 4-byte aligned for bf16 / 8 for float)
template <typename T, int N>
__device__ __forceinline__ void store_cos_sin(T *cp, T *sp, const float *vals, float scale) {
  if constexpr (sizeof(T) == 2 && N % 8 == 0) {
#pragma unroll
    for (int c = 0; c < N; c += 8) {
      uint32_t cw[4], sw[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float s0, c0, s1, c1;
        sincos_2pi_fast(vals[c + 2 * k] * scale, &s0, &c0);
        sincos_2pi_fast(vals[c + 2 * k + 1] * scale, &s1, &c1);
        cw[k] = pack_bf16_rne(c0, c1);
        sw[k] = pack_bf16_rne(s0, s1);
      }
      *reinterpret_cast<uint4 *>(cp + c) = make_uint4(cw[0], cw[1], cw[2], cw[3]);
      *reinterpret_cast<uint4 *>(sp + c) = make_uint4(sw[0], sw[1], sw[2], sw[3]);
    }
  } else {
#pragma unroll
    for (int c = 0; c < N; c += 2) {
      float s0, c0, s1, c1;
      sincos_2pi_fast(vals[c] * scale, &s0, &c0);
      sincos_2pi_fast(vals[c + 1] * scale, &s1, &c1);
      store_pair(cp + c, c0, c1);
      store_pair(sp + c, s0, s1);
    }
  }
}

// lane l's R consecutive values of the token row (16-byte loads; aligned by the launcher)
template <typename T, int R>
__device__ __forceinline__ void load_row_part(const T *xr, float (&v)[R]) {
  if constexpr (sizeof(T) == 2 && R % 8 == 0) {
#pragma unroll
    for (int r = 0; r < R; r += 8) {
      const uint4 q = *reinterpret_cast<const uint4 *>(xr + r);
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w[k]));
        v[r + 2 * k] = f.x;
        v[r + 2 * k + 1] = f.y;
      }
    }
  } else {
#pragma unroll
    for (int r = 0; r < R; ++r) v[r] = to_f32(xr[r]);
  }
}

// FWHT branch (natural Sylvester order, / sqrt(d)): cos / sin into z[0:d], z[d:2d].
// v holds lane l's values x[R l .. R l + R) and is overwritten.
template <typename T, int R>
__device__ __forceinline__ void features_fwht(float (&v)[R], T *__restrict__ zr, int lane) {
  constexpr int d = 32 * R;
#pragma unroll
  for (int len = 1; len < R; len <<= 1) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (!(r & len)) {
        const float u = v[r], w = v[r + len];
        v[r] = u + w;
        v[r + len] = u - w;
      }
    }
  }
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) {
    const bool hi = lane & m;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float p = __shfl_xor_sync(0xffffffffu, v[r], m);
      v[r] = hi ? p - v[r] : v[r] + p;
    }
  }
  store_cos_sin<T, R>(zr + R * lane, zr + d + R * lane, v, rsqrtf((float)d));
}

// DCT branch: cos / sin of the projections hdct into z[2d:3d], z[3d:4d].
template <typename T, int R>
__device__ __forceinline__ void features_dct(const float *hrow, T *__restrict__ zr, int lane) {
  constexpr int d = 32 * R;
  float v[R];
  const float *hr = hrow + R * lane;
#pragma unroll
  for (int r = 0; r < R; r += 4) {
    const float4 q = *reinterpret_cast<const float4 *>(hr + r);
    v[r] = q.x; v[r + 1] = q.y; v[r + 2] = q.z; v[r + 3] = q.w;
  }
  store_cos_sin<T, R>(zr + 2 * d + R * lane, zr + 3 * d + R * lane, v, 1.f);
}

// Recursive Haar branch into z[4d:5d], z[5d:6d]; hv holds lane l's values of x and is
// overwritten.  buf == nullptr: each level's outputs get their sin / cos on the lanes that
// hold the level (lane 0 also takes the last R alone), the fewest instructions in total
// (many tokens).  buf (d floats of shared memory): the outputs are staged there and every
// lane then takes R consecutive ones, so no lane computes more sin / cos than the other
// branches' lanes (few tokens: the branch's serial time is the critical path).
template <typename T, int R>
__device__ __forceinline__ void features_haar(float (&hv)[R], T *__restrict__ zr, int lane, float *buf) {
  constexpr int d = 32 * R;
  const float r2 = 0.70710678118654752f;
  // levels n = 32R .. 2R span nl = n / R lanes
#pragma unroll
  for (int nl = 32; nl >= 2; nl >>= 1) {
    const int half_l = nl >> 1;
    float hi[R / 2];
#pragma unroll
    for (int r = 0; r < R; r += 2) hi[r / 2] = (hv[r] - hv[r + 1]) * r2;
    if (lane < nl) {
      const int o = half_l * R + (R / 2) * lane;  // ho[n/2 + i], i = (R lane + r) / 2
      if (buf) {
#pragma unroll
        for (int i = 0; i < R / 2; i += 4)
          *reinterpret_cast<float4 *>(buf + o + i) = make_float4(hi[i], hi[i + 1], hi[i + 2], hi[i + 3]);
      } else {
        store_cos_sin<T, R / 2>(zr + 4 * d + o, zr + 5 * d + o, hi, 1.f);
      }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float p = __shfl_down_sync(0xffffffffu, hv[r], half_l);
      hv[r] = (hv[r] + p) * r2;
    }
  }
  // levels n = R .. 2 inside lane 0, then ho[0]
  if (lane == 0) {
    float ho[R];
#pragma unroll
    for (int n = R; n > 1; n >>= 1) {
      const int half = n >> 1;
#pragma unroll
      for (int i = 0; i < half; ++i) ho[half + i] = (hv[2 * i] - hv[2 * i + 1]) * r2;
      float lo[R / 2 > 0 ? R / 2 : 1];
#pragma unroll
      for (int i = 0; i < half; ++i) lo[i] = (hv[i] + hv[i + half]) * r2;
#pragma unroll
      for (int i = 0; i < half; ++i) hv[i] = lo[i];
    }
    ho[0] = hv[0];
    if (buf) {
#pragma unroll
      for (int i = 0; i < R; i += 4) *reinterpret_cast<float4 *>(buf + i) = make_float4(ho[i], ho[i + 1], ho[i + 2], ho[i + 3]);
    } else {
      store_cos_sin<T, R>(zr + 4 * d, zr + 5 * d, ho, 1.f);
    }
  }
  if (buf) {
    __syncwarp();
    float vals[R];
#pragma unroll
    for (int i = 0; i < R; i += 4) {
      const float4 q = *reinterpret_cast<const float4 *>(buf + R * lane + i);
      vals[i] = q.x; vals[i + 1] = q.y; vals[i + 2] = q.z; vals[i + 3] = q.w;
    }
    store_cos_sin<T, R>(zr + 4 * d + R * lane, zr + 5 * d + R * lane, vals, 1.f);
  }
}

template <typename T, int R>
__global__ void __launch_bounds__(256)
ffn_features_warp_kernel(const T *__restrict__ x, const float *__restrict__ hdct, T *__restrict__ z, int tokens) {
  // R >= 8: the 16-byte loads of x and hdct and the z stores of a lane start on 16-byte
  // boundaries, and the Haar output runs of a lane have an even length
  static_assert(R >= 8 && R % 8 == 0, "warp features need d = 256, 512 or 1024");
  constexpr int d = 32 * R;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= tokens) return;  // whole warps only: no block barrier in this kernel
  float v[R], hv[R];
  load_row_part<T, R>(x + row * d + R * lane, v);
#pragma unroll
  for (int r = 0; r < R; ++r) hv[r] = v[r];
  T *zr = z + row * 6 * d;
  features_fwht<T, R>(v, zr, lane);
  if (hdct) features_dct<T, R>(hdct + row * d, zr, lane);
  features_haar<T, R>(hv, zr, lane, nullptr);
}

// Few tokens (decode): one CTA of three warps per token, warp w computing branch w
// (FWHT, DCT, Haar) of the warp kernel above, so a token's features take a third of
// the serial time.
template <typename T, int R>
__global__ void __launch_bounds__(96)
ffn_features_split_kernel(const T *x, const float *hdct, T *__restrict__ z) {
  static_assert(R >= 8 && R % 8 == 0, "warp features need d = 256, 512 or 1024");
  constexpr int d = 32 * R;
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31, part = threadIdx.x >> 5;
  const int64_t row = blockIdx.x;
  T *zr = z + row * 6 * d;
  if (part == 1) {
    if (hdct) features_dct<T, R>(hdct + row * d, zr, lane);
    return;
  }
  __shared__ __align__(16) float haar_out[d];  // the Haar warp's staged outputs
  float v[R];
  load_row_part<T, R>(x + row * d + R * lane, v);
  if (part == 0)
    features_fwht<T, R>(v, zr, lane);
  else
    features_haar<T, R>(v, zr, lane, haar_out);
}

// ---------------------------------------------------------------- GEMM helpers
template <typename T>
__device__ __forceinline__ float ld_f32(const T *p, int64_t i) { return to_f32(p[i]); }

// C[m][n] (+)= sum_k A[m][k] B(k, n), B(k, n) = B[k ldb + n] or, if B_TRANS, B[n ldb + k]
// (ACC: added to C).  64 x 64 output tile per CTA, 4 x 4 per thread, fp32 accumulation:
// the CUDA-core GEMM for widths the tensor-core kernel does not take, and for the
// allocation-free entry point.
template <typename TA, typename TB, typename TC, bool B_TRANS, bool ACC = false>
__global__ void __launch_bounds__(256)
small_gemm_kernel(const TA *__restrict__ A, int lda, const TB *__restrict__ B, int ldb,
                  TC *__restrict__ C, int ldc, int M, int N, int K) {
  __shared__ float As[16][64 + 4];
  __shared__ float Bs[16][64 + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += 16) {
    for (int i = threadIdx.x; i < 64 * 16; i += 256) {
      const int m = i >> 4, k = i & 15;
      As[k][m] = (m0 + m < M && k0 + k < K) ? ld_f32(A, (int64_t)(m0 + m) * lda + k0 + k) : 0.f;
      int n, kb;
      if (B_TRANS) { n = i >> 4; kb = i & 15; } else { kb = i >> 6; n = i & 63; }
      float bv = 0.f;
      if (n0 + n < N && k0 + kb < K)
        bv = B_TRANS ? ld_f32(B, (int64_t)(n0 + n) * ldb + k0 + kb) : ld_f32(B, (int64_t)(k0 + kb) * ldb + n0 + n);
      Bs[kb][n] = bv;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = As[k][ty * 4 + i];
        b[i] = Bs[k][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int m = m0 + ty * 4 + i, n = n0 + tx * 4 + j;
      if (m < M && n < N) {
        const float prev = ACC ? to_f32(C[(int64_t)m * ldc + n]) : 0.f;
        C[(int64_t)m * ldc + n] = from_f32<TC>(prev + acc[i][j]);
      }
    }
}

// Ft (cols x rows) = F^T for F (rows x cols) row-major: 32 x 32 tiles through shared memory.
template <typename T>
__global__ void __launch_bounds__(256) transpose_kernel(const T *__restrict__ F, T *__restrict__ Ft, int rows,
                                                        int cols) {
  __shared__ T tile[32][33];
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32, tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int i = ty; i < 32; i += 8)
    if (r0 + i < rows && c0 + tx < cols) tile[i][tx] = F[(int64_t)(r0 + i) * cols + c0 + tx];
  __syncthreads();
  for (int i = ty; i < 32; i += 8)
    if (c0 + i < cols && r0 + tx < rows) Ft[(int64_t)(c0 + i) * rows + r0 + tx] = tile[tx][i];
}

}  // namespace
}  // namespace dp

extern "C" int dp_ffn_fold(const float *logits, const float *mats, const float *banks,
                           const float *combine, float *F, int d, int nb, void *stream) {
  using namespace dp;
  DP_REQUIRE(logits && mats && banks && combine && F, DP_ERR_INVALID_ARGUMENT, "dp_ffn_fold: null pointer");
  DP_REQUIRE(d >= 1 && nb >= 1, DP_ERR_INVALID_ARGUMENT, "dp_ffn_fold: bad sizes");
  const int nt = (d + kFoldTile - 1) / kFoldTile;
  dim3 grid(nt, nt, 6);
  ffn_fold_kernel<<<grid, kFoldTile * 8, 0, as_stream(stream)>>>(logits, mats, banks, combine, F, d, nb);
  return check_launch("ffn_fold_kernel");
}

namespace dp {
namespace {
// Workspace of dp_ffn_fwd: the DCT projections (tokens x d fp32), the features z
// (tokens x 6d, x's dtype) and F^T (d x 6d, x's dtype; the tensor-core GEMM reads both of
// its operands along K), each at a 256-byte boundary.
struct FfnWorkspace {
  size_t z_off, ft_off, total;
};
FfnWorkspace ffn_workspace_layout(int tokens, int d, int x_dtype) {
  const size_t es = dtype_size(x_dtype);
  auto up = [](size_t v) { return (v + 255) & ~(size_t)255; };
  FfnWorkspace w;
  w.z_off = up((size_t)tokens * d * sizeof(float));
  w.ft_off = w.z_off + up((size_t)tokens * 6 * d * es);
  w.total = w.ft_off + up((size_t)6 * d * d * es);
  return w;
}
}  // namespace
}  // namespace dp

extern "C" size_t dp_ffn_workspace_size(int tokens, int d, int x_dtype) {
  if (tokens <= 0 || d <= 0) return 0;
  return dp::ffn_workspace_layout(tokens, d, x_dtype).total;
}

namespace dp {
namespace {
// z (tokens, 6d) = the sin / cos features of x given its DCT projections hdct (tokens, d)
// float32; x, z of dtype bf16 (bf = true) or float32, hdct and z 16-byte aligned.  With
// hdct null the DCT branch's features are left alone (the DCT GEMM wrote them).
int launch_features(const void *x, bool bf, const float *hdct, void *z, int tokens, int d, cudaStream_t st) {
  int log2d = 0;
  while ((1 << log2d) < d) ++log2d;
  const size_t smem = 4 * (size_t)d * sizeof(float);
  const int threads = d >= 256 ? 256 : d;
  for (cudaError_t e : {cudaFuncSetAttribute(ffn_features_kernel<__nv_bfloat16>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                        cudaFuncSetAttribute(ffn_features_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem)})
    if (e != cudaSuccess) return set_error(DP_ERR_CUDA, std::string("ffn features smem attr: ") + cudaGetErrorString(e));
  const int wgrid = (tokens + 7) / 8;
  // below about one warp per SM sub-partition the three branches of a token run on
  // three warps (ffn_features_split_kernel); above, one warp per token
  const bool split = tokens <= kFeatSplitTokens;
  cudaError_t le = cudaSuccess;
  auto warp_features = [&](auto rc) {
    constexpr int R = decltype(rc)::value;
    if (bf && split)
      le = launch_pdl(ffn_features_split_kernel<__nv_bfloat16, R>, dim3(tokens), dim3(96), 0, st,
                      static_cast<const __nv_bfloat16 *>(x), hdct, static_cast<__nv_bfloat16 *>(z));
    else if (split)
      le = launch_pdl(ffn_features_split_kernel<float, R>, dim3(tokens), dim3(96), 0, st,
                      static_cast<const float *>(x), hdct, static_cast<float *>(z));
    else if (bf)
      ffn_features_warp_kernel<__nv_bfloat16, R><<<wgrid, 256, 0, st>>>(
          static_cast<const __nv_bfloat16 *>(x), hdct, static_cast<__nv_bfloat16 *>(z), tokens);
    else
      ffn_features_warp_kernel<float, R><<<wgrid, 256, 0, st>>>(static_cast<const float *>(x), hdct,
                                                                 static_cast<float *>(z), tokens);
  };
  const bool x16 = (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  if (!x16) {
    // unaligned rows: the block-per-token kernel below
  } else if (d == 1024) warp_features(std::integral_constant<int, 32>{});
  else if (d == 512) warp_features(std::integral_constant<int, 16>{});
  else if (d == 256) warp_features(std::integral_constant<int, 8>{});
  if (x16 && d >= 256 && d <= 1024) {
    // launched above
  } else if (bf)
    ffn_features_kernel<__nv_bfloat16><<<tokens, threads, smem, st>>>(
        static_cast<const __nv_bfloat16 *>(x), hdct, static_cast<__nv_bfloat16 *>(z), d, log2d);
  else
    ffn_features_kernel<float><<<tokens, threads, smem, st>>>(static_cast<const float *>(x), hdct,
                                                               static_cast<float *>(z), d, log2d);
  return pdl_status(le, "ffn_features_kernel");
}

// dp_ffn_fwd (accumulate = false: y = z F in x's dtype) and dp_ffn_fwd_residual
// (accumulate = true: y float32, y += z F in the combine GEMM's epilogue).
int ffn_fwd_impl(const void *x, int x_dtype, const void *dct, const void *F, void *y, int tokens, int d,
                 void *workspace, size_t workspace_bytes, void *stream, bool accumulate) {
  DP_REQUIRE(tokens >= 0 && d >= 1, DP_ERR_INVALID_ARGUMENT, "dp_ffn_fwd: bad sizes");
  DP_REQUIRE(x_dtype == DP_F32 || x_dtype == DP_BF16, DP_ERR_INVALID_ARGUMENT,
             "dp_ffn_fwd: x dtype must be float32 or bfloat16");
  DP_REQUIRE((d & (d - 1)) == 0 && d >= 8 && d <= 4096, DP_ERR_UNSUPPORTED,
             "dp_ffn_fwd: d must be a power of two in [8, 4096]");
  if (tokens == 0) return DP_OK;
  DP_REQUIRE(x && dct && F && y && workspace, DP_ERR_INVALID_ARGUMENT, "dp_ffn_fwd: null pointer");
  DP_REQUIRE(workspace_bytes >= dp_ffn_workspace_size(tokens, d, x_dtype), DP_ERR_WORKSPACE,
             "dp_ffn_fwd: workspace too small");
  DP_REQUIRE(reinterpret_cast<uintptr_t>(workspace) % 256 == 0, DP_ERR_MISALIGNED,
             "dp_ffn_fwd: workspace must be 256-byte aligned");
  cudaStream_t st = as_stream(stream);
  const FfnWorkspace wl = ffn_workspace_layout(tokens, d, x_dtype);
  float *hdct = static_cast<float *>(workspace);
  void *z = static_cast<char *>(workspace) + wl.z_off;
  void *Ft = static_cast<char *>(workspace) + wl.ft_off;
  const bool bf = x_dtype == DP_BF16;
  const int es = bf ? 2 : 4;
  // z and F^T sit at 256-byte boundaries of the workspace; x and dct must be 16-byte aligned
  const bool tc = gemm_tc_supported(es, x, dct, tokens, d, d, d, d, 128) &&
                  gemm_tc_supported(es, workspace, workspace, tokens, d, 6 * d, 6 * d, 6 * d);
  if (tc) {
    // tcgen05 GEMMs (bf16, or fp32 read as tf32): Hdct = X Cdct^T, then Y (+)= Z F with F^T
    // formed in the workspace.  For bf16 the DCT GEMM's epilogue writes the DCT branch's
    // cos / sin into z itself (blocks 2 and 3 of each row), so the projections never reach
    // HBM and the feature kernel computes the FWHT and Haar branches only.
    int rc;
    if (bf) {
      rc = gemm_tc(es, x, d, dct, d, static_cast<__nv_bfloat16 *>(z) + 2 * d, 6 * d, tokens, d, d, 3, st, d, 128);
      if (rc != DP_OK) return rc;
      rc = launch_features(x, bf, nullptr, z, tokens, d, st);
    } else {
      rc = gemm_tc(es, x, d, dct, d, hdct, d, tokens, d, d, 0, st);
      if (rc != DP_OK) return rc;
      rc = launch_features(x, bf, hdct, z, tokens, d, st);
    }
    if (rc != DP_OK) return rc;
    dim3 tg((d + 31) / 32, (6 * d + 31) / 32);
    if (bf)
      transpose_kernel<__nv_bfloat16><<<tg, 256, 0, st>>>(static_cast<const __nv_bfloat16 *>(F),
                                                          static_cast<__nv_bfloat16 *>(Ft), 6 * d, d);
    else
      transpose_kernel<float><<<tg, 256, 0, st>>>(static_cast<const float *>(F), static_cast<float *>(Ft), 6 * d, d);
    rc = check_launch("transpose_kernel");
    if (rc != DP_OK) return rc;
    return gemm_tc(es, z, 6 * d, Ft, 6 * d, y, d, tokens, d, 6 * d, accumulate ? 2 : (bf ? 1 : 0), st);
  }
  // widths the tensor-core kernel does not take (d < 64): the CUDA-core GEMM
  dim3 g1((d + 63) / 64, (tokens + 63) / 64);
  dim3 g2((d + 63) / 64, (tokens + 63) / 64);
  int rc;
  if (bf) {
    small_gemm_kernel<__nv_bfloat16, __nv_bfloat16, float, true><<<g1, 256, 0, st>>>(
        static_cast<const __nv_bfloat16 *>(x), d, static_cast<const __nv_bfloat16 *>(dct), d, hdct, d, tokens, d, d);
  } else {
    small_gemm_kernel<float, float, float, true><<<g1, 256, 0, st>>>(static_cast<const float *>(x), d,
                                                                      static_cast<const float *>(dct), d, hdct, d,
                                                                      tokens, d, d);
  }
  rc = check_launch("small_gemm_kernel (DCT)");
  if (rc != DP_OK) return rc;
  rc = launch_features(x, bf, hdct, z, tokens, d, st);
  if (rc != DP_OK) return rc;
  if (accumulate) {
    if (bf)
      small_gemm_kernel<__nv_bfloat16, __nv_bfloat16, float, false, true><<<g2, 256, 0, st>>>(
          static_cast<const __nv_bfloat16 *>(z), 6 * d, static_cast<const __nv_bfloat16 *>(F), d,
          static_cast<float *>(y), d, tokens, d, 6 * d);
    else
      small_gemm_kernel<float, float, float, false, true><<<g2, 256, 0, st>>>(
          static_cast<const float *>(z), 6 * d, static_cast<const float *>(F), d, static_cast<float *>(y), d, tokens,
          d, 6 * d);
  } else if (bf) {
    small_gemm_kernel<__nv_bfloat16, __nv_bfloat16, __nv_bfloat16, false><<<g2, 256, 0, st>>>(
        static_cast<const __nv_bfloat16 *>(z), 6 * d, static_cast<const __nv_bfloat16 *>(F), d,
        static_cast<__nv_bfloat16 *>(y), d, tokens, d, 6 * d);
  } else {
    small_gemm_kernel<float, float, float, false><<<g2, 256, 0, st>>>(
        static_cast<const float *>(z), 6 * d, static_cast<const float *>(F), d, static_cast<float *>(y), d, tokens,
        d, 6 * d);
  }
  return check_launch("small_gemm_kernel (combine)");
}
}  // namespace
}  // namespace dp

extern "C" int dp_ffn_fwd(const void *x, int x_dtype, const void *dct, const void *F, void *y,
                          int tokens, int d, void *workspace, size_t workspace_bytes, void *stream) {
  return dp::ffn_fwd_impl(x, x_dtype, dct, F, y, tokens, d, workspace, workspace_bytes, stream, false);
}

extern "C" int dp_ffn_fwd_residual(const void *x, int x_dtype, const void *dct, const void *F, float *y,
                                   int tokens, int d, void *workspace, size_t workspace_bytes, void *stream) {
  return dp::ffn_fwd_impl(x, x_dtype, dct, F, y, tokens, d, workspace, workspace_bytes, stream, true);
}

// ---------------------------------------------------------------------------------
// Allocation-free FFN forward (dp_ffn_fwd_noalloc).
//
// Some callers cannot allocate device memory where they run the FFN: code being
// captured into a CUDA graph (cudaMalloc is not a capturable operation), host runtimes
// that hand the whole device heap to their own allocator and forbid any other
// allocation, and latency-bound decode loops that must never block on the driver's
// allocator.  This entry point takes its scratch -- the DCT projections and the
// sin/cos features of the tokens -- from the fixed array below, which lives in the
// library's device image, and it runs its two GEMMs with a CUDA-core kernel of this
// file (the tensor-core path of dp_ffn_fwd needs workspace for F^T).
//
// The array is kFfnScratchBytes on every GPU that loads the library, held until the
// process exits.  All calls share it and it keeps the last call's contents; nothing in
// it has to start at zero (every scratch element a call reads is written by that call
// first), but calls that overlap on the GPU -- concurrent streams, or another host
// thread -- race on it and must be serialised by the caller.
static __device__ __align__(256) unsigned char g_ffn_scratch[8u << 20];

namespace dp {
namespace {

constexpr size_t kFfnScratchBytes = 8u << 20;

// Device address of g_ffn_scratch on the current device, looked up on every call with
// that device current (the lookup allocates nothing; not caching it keeps it right after
// a device reset, which can move the array).  The first call on a device also loads
// every kernel this entry point can launch, for both dtypes: CUDA loads kernel code
// lazily on first launch, and loading is itself a device allocation, so after this
// first call no later call loads anything.
int ffn_scratch_address(void **out) {
  static std::mutex mu;
  static bool loaded[64] = {false};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(DP_ERR_CUDA, std::string("dp_ffn_fwd_noalloc: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return set_error(DP_ERR_UNSUPPORTED, "dp_ffn_fwd_noalloc: device ordinal >= 64");
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!loaded[dev]) {
      const void *kernels[6] = {
          reinterpret_cast<const void *>(small_gemm_kernel<float, float, float, true>),
          reinterpret_cast<const void *>(small_gemm_kernel<float, float, float, false>),
          reinterpret_cast<const void *>(small_gemm_kernel<__nv_bfloat16, __nv_bfloat16, float, true>),
          reinterpret_cast<const void *>(small_gemm_kernel<__nv_bfloat16, __nv_bfloat16, __nv_bfloat16, false>),
          reinterpret_cast<const void *>(ffn_features_kernel<float>),
          reinterpret_cast<const void *>(ffn_features_kernel<__nv_bfloat16>)};
      for (const void *k : kernels) {
        cudaFuncAttributes attr;
        e = cudaFuncGetAttributes(&attr, k);
        if (e != cudaSuccess)
          return set_error(DP_ERR_CUDA, std::string("dp_ffn_fwd_noalloc: kernel load failed: ") +
                                            cudaGetErrorString(e));
      }
      loaded[dev] = true;
    }
  }
  void *p = nullptr;
  e = cudaGetSymbolAddress(&p, g_ffn_scratch);
  if (e != cudaSuccess || p == nullptr)
    return set_error(DP_ERR_CUDA, std::string("dp_ffn_fwd_noalloc: cudaGetSymbolAddress failed: ") +
                                      cudaGetErrorString(e));
  *out = p;
  return DP_OK;
}

template <typename T>
int ffn_fwd_noalloc_typed(const T *x, const T *dct, const T *F, T *y, int tokens, int d,
                          unsigned char *scratch, cudaStream_t st) {
  float *hdct = reinterpret_cast<float *>(scratch);
  T *z = reinterpret_cast<T *>(scratch + (((size_t)tokens * d * sizeof(float) + 255) & ~(size_t)255));
  dim3 g1((d + 63) / 64, (tokens + 63) / 64);
  small_gemm_kernel<T, T, float, true><<<g1, 256, 0, st>>>(x, d, dct, d, hdct, d, tokens, d, d);
  int rc = check_launch("small_gemm_kernel (DCT)");
  if (rc != DP_OK) return rc;
  int log2d = 0;
  while ((1 << log2d) < d) ++log2d;
  const size_t smem = 4 * (size_t)d * sizeof(float);
  cudaError_t e = cudaFuncSetAttribute(ffn_features_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess)
    return set_error(DP_ERR_CUDA, std::string("ffn features smem attr: ") + cudaGetErrorString(e));
  ffn_features_kernel<T><<<tokens, d >= 256 ? 256 : d, smem, st>>>(x, hdct, z, d, log2d);
  rc = check_launch("ffn_features_kernel");
  if (rc != DP_OK) return rc;
  dim3 g2((d + 63) / 64, (tokens + 63) / 64);
  small_gemm_kernel<T, T, T, false><<<g2, 256, 0, st>>>(z, 6 * d, F, d, y, d, tokens, d, 6 * d);
  return check_launch("small_gemm_kernel (combine)");
}

}  // namespace
}  // namespace dp

extern "C" size_t dp_ffn_noalloc_max_tokens(int d, int x_dtype) {
  if (d <= 0 || !(x_dtype == DP_F32 || x_dtype == DP_BF16)) return 0;
  const size_t per_token = (size_t)d * sizeof(float) + (size_t)6 * d * dp::dtype_size(x_dtype);
  return (dp::kFfnScratchBytes - 256) / per_token;
}

extern "C" int dp_ffn_fwd_noalloc(const void *x, int x_dtype, const void *dct, const void *F, void *y,
                                  int tokens, int d, void *stream) {
  using namespace dp;
  DP_REQUIRE(tokens >= 0 && d >= 1, DP_ERR_INVALID_ARGUMENT, "dp_ffn_fwd_noalloc: bad sizes");
  DP_REQUIRE(x_dtype == DP_F32 || x_dtype == DP_BF16, DP_ERR_INVALID_ARGUMENT,
             "dp_ffn_fwd_noalloc: x dtype must be float32 or bfloat16");
  DP_REQUIRE((d & (d - 1)) == 0 && d >= 8 && d <= 4096, DP_ERR_UNSUPPORTED,
             "dp_ffn_fwd_noalloc: d must be a power of two in [8, 4096]");
  const size_t max_tokens = dp_ffn_noalloc_max_tokens(d, x_dtype);
  if ((size_t)tokens > max_tokens)
    return set_error(DP_ERR_WORKSPACE,
                     "dp_ffn_fwd_noalloc: " + std::to_string(tokens) + " tokens exceed the 8 MiB static "
                     "scratch (at most " + std::to_string(max_tokens) + " tokens at d=" + std::to_string(d) +
                     "); call dp_ffn_fwd with a workspace, or split the tokens");
  if (tokens == 0) return DP_OK;
  DP_REQUIRE(x && dct && F && y, DP_ERR_INVALID_ARGUMENT, "dp_ffn_fwd_noalloc: null pointer");
  void *scratch = nullptr;
  int rc = ffn_scratch_address(&scratch);
  if (rc != DP_OK) return rc;
  unsigned char *sp = static_cast<unsigned char *>(scratch);
  cudaStream_t st = as_stream(stream);
  if (x_dtype == DP_BF16)
    return ffn_fwd_noalloc_typed(static_cast<const __nv_bfloat16 *>(x), static_cast<const __nv_bfloat16 *>(dct),
                                 static_cast<const __nv_bfloat16 *>(F), static_cast<__nv_bfloat16 *>(y), tokens,
                                 d, sp, st);
  return ffn_fwd_noalloc_typed(static_cast<const float *>(x), static_cast<const float *>(dct),
                               static_cast<const float *>(F), static_cast<float *>(y), tokens, d, sp, st);
}

extern "C" int dp_ffn_features(const void *x, int x_dtype, const float *hdct, void *z, int tokens, int d,
                               void *stream) {
  using namespace dp;
  DP_REQUIRE(tokens >= 0 && d >= 1, DP_ERR_INVALID_ARGUMENT, "dp_ffn_features: bad sizes");
  DP_REQUIRE(x_dtype == DP_F32 || x_dtype == DP_BF16, DP_ERR_INVALID_ARGUMENT,
             "dp_ffn_features: x dtype must be float32 or bfloat16");
  DP_REQUIRE((d & (d - 1)) == 0 && d >= 8 && d <= 4096, DP_ERR_UNSUPPORTED,
             "dp_ffn_features: d must be a power of two in [8, 4096]");
  if (tokens == 0) return DP_OK;
  DP_REQUIRE(x && hdct && z, DP_ERR_INVALID_ARGUMENT, "dp_ffn_features: null pointer");
  DP_REQUIRE(reinterpret_cast<uintptr_t>(hdct) % 16 == 0 && reinterpret_cast<uintptr_t>(z) % 16 == 0,
             DP_ERR_MISALIGNED, "dp_ffn_features: hdct and z must be 16-byte aligned");
  return launch_features(x, x_dtype == DP_BF16, hdct, z, tokens, d, as_stream(stream));
}
