// Shared helpers of the deltaphase_b200 CUDA library (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <string>

#include "../../include/deltaphase_b200.h"

namespace dp {

// ---------------------------------------------------------------- errors
// Records the message of the last failed call for the calling host thread.
int set_error(int status, const std::string &msg);
int check_launch(const char *what);

#define DP_REQUIRE(cond, status, msg)                  \
  do {                                                 \
    if (!(cond)) return ::dp::set_error((status), (msg)); \
  } while (0)

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

// ---------------------------------------------------------------- dependent launch
// The token-step kernels run back to back, each a few microseconds long, so the gap
// between two launches is a large part of a step.  They are launched with programmatic
// dependent launch: a kernel may start while its predecessor in the stream still runs,
// and waits in pdl_wait() (griddepcontrol.wait: until the predecessor grid has completed
// and its writes are visible) before it touches memory that earlier kernels write, or
// writes memory they read.  Right after its wait it lets its own successor start
// (pdl_trigger).  Without the launch attribute both instructions do nothing.
// Data written by earlier kernels is read with coherent loads in these kernels (no
// __ldg, no const __restrict__ on those pointers): the read-only path assumes memory that
// stays fixed for the kernel's lifetime, which a kernel started early does not see.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

// kern<<<grid, block, smem, st>>>(args...) with the programmatic-dependent-launch
// attribute; returns the launch status.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// Ask the L2 to fetch `bytes` (a multiple of 16) from p (16-byte aligned): a TMA bulk
// prefetch, which needs no registers and no completion wait.  Safe before pdl_wait: it
// returns no data to the thread, and the L2 is coherent with the writes of other kernels.
__device__ __forceinline__ void prefetch_l2_bulk(const void *p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(p), "r"(bytes) : "memory");
}

// The same for an arbitrary span: the 16-byte aligned interior of [p, p + bytes).
__device__ __forceinline__ void prefetch_l2_span(const void *p, size_t bytes) {
  const uintptr_t a = (reinterpret_cast<uintptr_t>(p) + 15) & ~uintptr_t(15);
  const uintptr_t e = (reinterpret_cast<uintptr_t>(p) + bytes) & ~uintptr_t(15);
  if (e > a) prefetch_l2_bulk(reinterpret_cast<const void *>(a), (uint32_t)(e - a));
}

// Status of a launch_pdl call (DP_OK, or DP_ERR_CUDA with the message recorded).
inline int pdl_status(cudaError_t e, const char *what) {
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(DP_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  }
  return check_launch(what);
}

// ---------------------------------------------------------------- dtypes
template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <>
__device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

// Scalar of runtime dtype dt, loaded as raw bits and converted later: a prefetch whose
// value is needed only after other work must not convert at the load (the conversion
// would wait for the load).
__device__ __forceinline__ uint32_t load_raw_scalar(const void *p, int dt, int64_t i) {
  if (dt == DP_F32) return __ldg(static_cast<const unsigned int *>(p) + i);
  return __ldg(static_cast<const unsigned short *>(p) + i);
}
__device__ __forceinline__ float raw_scalar_to_f32(uint32_t raw, int dt) {
  if (dt == DP_F32) return __uint_as_float(raw);
  if (dt == DP_BF16) return __uint_as_float(raw << 16);
  return __half2float(__ushort_as_half(static_cast<unsigned short>(raw)));
}

inline bool valid_dtype(int dt) { return dt == DP_F32 || dt == DP_BF16 || dt == DP_F16; }
inline size_t dtype_size(int dt) { return dt == DP_F32 ? 4 : 2; }

// Calls f.template operator()<T>() with T the C++ type of dtype code dt.
template <typename F>
int dispatch_dtype(int dt, F &&f) {
  switch (dt) {
    case DP_F32: return f(float{});
    case DP_BF16: return f(__nv_bfloat16{});
    case DP_F16: return f(__half{});
    default: return set_error(DP_ERR_INVALID_ARGUMENT, "unknown dtype code");
  }
}

// Phase -> (cos, sin) with CUDA's accurate sincosf, for every input type (the CUDA-core
// kernels; the tensor-core kernels reduce the phase themselves and use the hardware
// approximation, see fast_sincos below).
template <typename T>
__device__ __forceinline__ void phase_sincos(T th, float *s, float *c) {
  sincosf(to_f32(th), s, c);
}

// sin and cos of x on the FMA pipe (no special-function unit): Cody-Waite reduction
// x = k pi/2 + r, |r| <= pi/4 (pi/2 split in a float head and tail), Taylor series of
// sin (to r^7) and cos (to r^8) on the reduced argument, quadrant fix-up from k mod 4.
// Truncation error < 4e-7 on |r| <= pi/4; max abs error ~2e-6 for |x| <= 20 (the
// reduction's rounding grows with |x|).
__device__ __forceinline__ void poly_sincos(float x, float *s_out, float *c_out) {
  const float kf = fmaf(x, 0.63661977236758134f, 12582912.0f);  // 1.5 * 2^23 rounds k
  const float k = kf - 12582912.0f;
  const int q = __float_as_int(kf);
  float r = fmaf(-k, 1.5707963705062866f, x);
  r = fmaf(-k, -4.371138828673793e-08f, r);
  const float r2 = r * r;
  float ps = fmaf(r2, -1.9841270113829523e-04f, 8.3333337679505348e-03f);
  ps = fmaf(r2, ps, -0.16666667163372040f);
  const float sn = fmaf(r * r2, ps, r);
  float pc = fmaf(r2, 2.4801587642286904e-05f, -1.3888889225199819e-03f);
  pc = fmaf(r2, pc, 4.1666667908430100e-02f);
  pc = fmaf(r2, pc, -0.5f);
  const float cs = fmaf(r2, pc, 1.0f);
  const bool swap = q & 1;
  float so = swap ? cs : sn, co = swap ? sn : cs;
  so = __uint_as_float(__float_as_uint(so) ^ (((unsigned)q & 2u) << 30));
  co = __uint_as_float(__float_as_uint(co) ^ (((unsigned)(q + 1) & 2u) << 30));
  *s_out = so;
  *c_out = co;
}

// sin and cos of x: x reduced by a two-part 2 pi to |r| <= pi, then the hardware
// approximation (absolute error ~1e-6 for |x| up to a few hundred) -- for values that are
// rounded to 16 bits or feed a TF32 / bf16 product next.
__device__ __forceinline__ void sincos_2pi_fast(float x, float *s, float *c) {
  // round x / 2 pi to an integer with the 1.5 * 2^23 add (FMA pipe; |x| < 2^22)
  const float k = fmaf(x, 0.15915494309189535f, 12582912.0f) - 12582912.0f;
  float r = fmaf(-k, 6.28318548202514648f, x);
  r = fmaf(-k, -1.7484556e-07f, r);
  __sincosf(r, s, c);
}

// Two floats -> packed bf16 pair, round to nearest even, with integer operations
// (finite inputs; keeps the conversion off the special-function pipe).
__device__ __forceinline__ uint32_t pack_bf16_rne(float a, float b) {
  uint32_t ua = __float_as_uint(a), ub = __float_as_uint(b);
  ua += 0x7FFFu + ((ua >> 16) & 1u);
  ub += 0x7FFFu + ((ub >> 16) & 1u);
  return __byte_perm(ua, ub, 0x7632);
}

struct SeqStrides {  // element strides of a (B, H, L, C) tensor with unit channel stride
  int64_t b, h, t;
};

}  // namespace dp
