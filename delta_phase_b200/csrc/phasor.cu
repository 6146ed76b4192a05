// Phasor generation e^{i theta} (interleaved complex64), the elementwise step of
// delta_phase/layers.py:203-206 and delta_phase/kernels/triton_chunk_delta.py:220-221
// (K = cos theta + i sin theta), computed with the FMA-pipe sin/cos of dp_common.cuh.
#include <algorithm>

#include "dp_common.cuh"

namespace dp {
namespace {

template <typename T>
__global__ void __launch_bounds__(256) phasor_kernel(const T *__restrict__ th, float2 *__restrict__ out, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float s, c;
    poly_sincos(to_f32(th[i]), &s, &c);
    out[i] = make_float2(c, s);
  }
}

}  // namespace
}  // namespace dp

extern "C" int dp_phasor(const void *theta, int dtype, int64_t n, float *out, void *stream) {
  using namespace dp;
  DP_REQUIRE(n >= 0, DP_ERR_INVALID_ARGUMENT, "dp_phasor: negative size");
  DP_REQUIRE(valid_dtype(dtype), DP_ERR_INVALID_ARGUMENT, "dp_phasor: bad dtype code");
  if (n == 0) return DP_OK;
  DP_REQUIRE(theta && out, DP_ERR_INVALID_ARGUMENT, "dp_phasor: null pointer");
  DP_REQUIRE((reinterpret_cast<uintptr_t>(out) & 7) == 0, DP_ERR_MISALIGNED, "dp_phasor: out must be 8-byte aligned");
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 148 * 16);
  return dispatch_dtype(dtype, [&](auto tag) -> int {
    using T = decltype(tag);
    phasor_kernel<T><<<blocks, 256, 0, as_stream(stream)>>>(static_cast<const T *>(theta),
                                                            reinterpret_cast<float2 *>(out), n);
    return check_launch("phasor_kernel");
  });
}
