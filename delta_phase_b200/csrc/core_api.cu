// dp_core_fwd: argument checks and kernel selection for the chunkwise core.
#include "dp_common.cuh"

namespace dp {
bool core_tc_supported(const void *tk, const void *tq, const void *v, int in_dt, const float *out,
                       int D, int Dv, const SeqStrides *s);
int core_fwd_tc(const void *tk, const void *tq, const void *v, const void *beta, int beta_dt,
                const float *state_in, float *out, float *state_out, int B, int H, int L,
                const SeqStrides *s, cudaStream_t stream, bool cbeta);
int core_fwd_simt(const void *tk, const void *tq, const void *v, const void *beta, int in_dt,
                  int beta_dt, const float *state_in, float *out, float *state_out, int B, int H,
                  int L, int D, int Dv, const SeqStrides *s, cudaStream_t stream, bool cbeta);

namespace {
// Shared by dp_core_fwd (beta real) and dp_core_cbeta_fwd (beta = 1 + e^{i phi}, `beta`
// holding phi): the argument checks and the kernel choice are the same.
int core_fwd_entry(const char *name, bool cbeta, const void *theta_k, const void *theta_q, const void *v,
                   const void *beta, int in_dtype, int beta_dtype, const float *state_in, float *out,
                   float *state_out, int B, int H, int L, int D, int Dv, int chunk_size,
                   const int64_t *strides, void *stream) {
  const std::string n(name);
  DP_REQUIRE(B >= 0 && H >= 0 && L >= 0, DP_ERR_INVALID_ARGUMENT, n + ": negative size");
  DP_REQUIRE(chunk_size >= 1, DP_ERR_INVALID_ARGUMENT, n + ": chunk_size must be >= 1");
  DP_REQUIRE(D >= 1 && Dv >= 1, DP_ERR_INVALID_ARGUMENT, n + ": D and Dv must be >= 1");
  DP_REQUIRE(D <= 128 && Dv <= 128, DP_ERR_UNSUPPORTED, n + ": D and Dv must be <= 128");
  DP_REQUIRE(valid_dtype(in_dtype) && valid_dtype(beta_dtype), DP_ERR_INVALID_ARGUMENT, n + ": bad dtype code");
  if (B == 0 || H == 0) return DP_OK;
  DP_REQUIRE(state_out && strides, DP_ERR_INVALID_ARGUMENT, n + ": null state_out/strides");
  DP_REQUIRE(L == 0 || (theta_k && theta_q && v && beta && out), DP_ERR_INVALID_ARGUMENT,
             n + ": null input pointer");
  SeqStrides s[5];
  for (int i = 0; i < 5; ++i) s[i] = SeqStrides{strides[3 * i], strides[3 * i + 1], strides[3 * i + 2]};
  if (core_tc_supported(theta_k, theta_q, v, in_dtype, out, D, Dv, s))
    return core_fwd_tc(theta_k, theta_q, v, beta, beta_dtype, state_in, out, state_out, B, H, L, s,
                       as_stream(stream), cbeta);
  return core_fwd_simt(theta_k, theta_q, v, beta, in_dtype, beta_dtype, state_in, out, state_out,
                       B, H, L, D, Dv, s, as_stream(stream), cbeta);
}
}  // namespace
}  // namespace dp

extern "C" int dp_core_fwd(const void *theta_k, const void *theta_q, const void *v,
                           const void *beta, int in_dtype, int beta_dtype, const float *state_in,
                           float *out, float *state_out, int B, int H, int L, int D, int Dv,
                           int chunk_size, const int64_t *strides, void *stream) {
  return dp::core_fwd_entry("dp_core_fwd", false, theta_k, theta_q, v, beta, in_dtype, beta_dtype, state_in, out,
                            state_out, B, H, L, D, Dv, chunk_size, strides, stream);
}

extern "C" int dp_core_cbeta_fwd(const void *theta_k, const void *theta_q, const void *v,
                                 const void *phi, int in_dtype, int phi_dtype, const float *state_in,
                                 float *out, float *state_out, int B, int H, int L, int D, int Dv,
                                 int chunk_size, const int64_t *strides, void *stream) {
  return dp::core_fwd_entry("dp_core_cbeta_fwd", true, theta_k, theta_q, v, phi, in_dtype, phi_dtype, state_in,
                            out, state_out, B, H, L, D, Dv, chunk_size, strides, stream);
}
