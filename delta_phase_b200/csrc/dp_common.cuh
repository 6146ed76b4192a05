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

// Phase -> (cos, sin).  float inputs use the accurate sincosf; 16-bit inputs use
// the hardware approximation, whose error (~1e-6 on [-pi, pi] after CUDA's own
// reduction) is far below the 16-bit input quantisation.
template <typename T>
__device__ __forceinline__ void phase_sincos(T th, float *s, float *c) {
  sincosf(to_f32(th), s, c);
}

struct SeqStrides {  // element strides of a (B, H, L, C) tensor with unit channel stride
  int64_t b, h, t;
};

}  // namespace dp
