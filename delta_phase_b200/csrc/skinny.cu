// Skinny GEMM for decode batches: y (M x N) = x (M x K) W^T (+ bias) (+ y), M <= 16.
//
// A decode step multiplies at most a few dozen token rows by each weight matrix, so the
// product is bound by reading W once from HBM (2 N K bytes in bf16), not by arithmetic:
// the input projections, out_proj, the FFN's DCT and folded-combine matrices of every
// block (delta_phase/layers.py:265-290, 119-141).  Library GEMMs tile M in 64- or
// 128-row blocks and leave most SMs idle at these shapes; this kernel spreads W over the
// whole GPU instead.
//
// Layout: x (M, K) and W (N, K) bf16 row-major (W in nn.Linear's layout), fp32
// accumulation on the m16n8k16 tensor-core MMA (M = 16 is one MMA tile; the kernel is
// HBM-bound, so the MMA's issue rate is not the limit).  Each warp owns 8 output columns
// and a K range; per 32-wide K step a lane loads one 16-byte run of 8 consecutive k of
// its W row and of its two x rows, and feeds them to two MMAs through a fixed permutation
// of the k slots (the same for A and B, so the dot products are unchanged).  The K range
// is split over the KS CTAs (up to 16) of a thread-block cluster, chosen so the grid is
// one wave; the partial tiles are summed through distributed shared memory in a fixed
// rank order (deterministic), and the epilogue adds the bias and, optionally, the
// existing y.  Launched as a dependent launch (dp_common.cuh): the CTAs start fetching
// their weight slices into L2 while the previous kernel of the step still runs.
#include <cooperative_groups.h>

#include <string>

#include "dp_common.cuh"

namespace cg = cooperative_groups;

namespace dp {
namespace {

constexpr int kSkWarps = 4;             // warps per CTA
constexpr int kSkCols = kSkWarps * 8;    // output columns per CTA
constexpr int kSkUnr = 2;               // K steps per load batch
constexpr int kSkWaveCtas = 148 * 8;    // CTAs of one wave (8 per SM)

__device__ __forceinline__ void mma_16816_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float load_scalar(const void *p, int dt, int64_t i) {
  if (dt == DP_F32) return static_cast<const float *>(p)[i];
  if (dt == DP_BF16) return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
  return __half2float(static_cast<const __half *>(p)[i]);
}

__device__ __forceinline__ void store_scalar(void *p, int dt, int64_t i, float v) {
  if (dt == DP_F32)
    static_cast<float *>(p)[i] = v;
  else if (dt == DP_BF16)
    static_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v);
  else
    static_cast<__half *>(p)[i] = __float2half_rn(v);
}

// One 32-wide K step of a warp: x rows g, g + 8 and W row n, 8 consecutive k per lane.
struct SkStep {
  uint4 a, b, w;
};

__device__ __forceinline__ void sk_load(SkStep &s, const __nv_bfloat16 *x0, const __nv_bfloat16 *x1,
                                        const __nv_bfloat16 *wr, int k) {
  s.a = *reinterpret_cast<const uint4 *>(x0 + k);  // coherent loads: x may come from the
  s.b = *reinterpret_cast<const uint4 *>(x1 + k);  // kernel this one overlaps (pdl_wait)
  s.w = __ldcs(reinterpret_cast<const uint4 *>(wr + k));
}

// k slots {2t, 2t+1 | 2t+8, 2t+9} hold k = {8t, 8t+1 | 8t+2, 8t+3} in the first MMA and
// {8t+4, 8t+5 | 8t+6, 8t+7} in the second
__device__ __forceinline__ void sk_mma(float (&acc)[4], const SkStep &s) {
  mma_16816_bf16(acc, s.a.x, s.b.x, s.a.y, s.b.y, s.w.x, s.w.y);
  mma_16816_bf16(acc, s.a.z, s.b.z, s.a.w, s.b.w, s.w.z, s.w.w);
}

// Grid (KS, ceil(N / kSkCols)), cluster (KS, 1, 1): blockIdx.x is the K split (the CTA's
// rank in its cluster), blockIdx.y the column tile.  Each warp owns 8 columns; its K
// range streams in batches of kSkUnr steps, the next batch's loads issued before the
// current batch's MMAs (register double buffering).
template <int KS>
__global__ void __launch_bounds__(kSkWarps * 32)
skinny_gemm_kernel(const __nv_bfloat16 *x, int64_t ldx, const __nv_bfloat16 *__restrict__ w,
                   const void *__restrict__ bias, int bias_dt, void *y, int y_dt, int64_t ldy, int accumulate,
                   int M, int N, int K) {
  __shared__ float part[16 * kSkCols];  // this CTA's partial (16, kSkCols) tile
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int n_cta = blockIdx.y * kSkCols;
  const int k_per = K / KS;  // a multiple of 32 (checked by the launcher)
  // the weights do not depend on earlier kernels: start their fetch into L2 before
  // waiting for the predecessor (the CTA's 32 row segments of k_per values)
  if (warp == 0 && n_cta + lane < N)
    prefetch_l2_bulk(w + (int64_t)(n_cta + lane) * K + rank * k_per, (uint32_t)k_per * 2u);
  pdl_wait();
  pdl_trigger();
  const int k0 = rank * k_per + 8 * t;
  // rows >= M and columns >= N read a valid row (M - 1, N - 1) and are not stored
  const __nv_bfloat16 *x0 = x + (int64_t)min(g, M - 1) * ldx + k0;
  const __nv_bfloat16 *x1 = x + (int64_t)min(g + 8, M - 1) * ldx + k0;
  const __nv_bfloat16 *wr = w + (int64_t)min(n_cta + warp * 8 + g, N - 1) * K + k0;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  SkStep cur[kSkUnr], nxt[kSkUnr];
#pragma unroll
  for (int u = 0; u < kSkUnr; ++u)
    if (32 * u < k_per) sk_load(cur[u], x0, x1, wr, 32 * u);  // conditions uniform over the warp
  for (int k = 0; k < k_per; k += 32 * kSkUnr) {
    const int kn = k + 32 * kSkUnr;
#pragma unroll
    for (int u = 0; u < kSkUnr; ++u)
      if (kn + 32 * u < k_per) sk_load(nxt[u], x0, x1, wr, kn + 32 * u);
#pragma unroll
    for (int u = 0; u < kSkUnr; ++u)
      if (k + 32 * u < k_per) sk_mma(acc, cur[u]);
#pragma unroll
    for (int u = 0; u < kSkUnr; ++u) cur[u] = nxt[u];
  }
  // accumulator: rows g / g + 8, columns 2t, 2t + 1 of the warp's 8 columns
  const int c = warp * 8 + 2 * t;
  part[g * kSkCols + c] = acc[0];
  part[g * kSkCols + c + 1] = acc[1];
  part[(g + 8) * kSkCols + c] = acc[2];
  part[(g + 8) * kSkCols + c + 1] = acc[3];
  cluster.sync();
  // rank r sums its share of the tile over the KS partials, in rank order
  constexpr int kElems = 16 * kSkCols;
  constexpr int kPer = (kElems + KS - 1) / KS;
  const int e_end = min(kElems, (rank + 1) * kPer);
  for (int e = rank * kPer + threadIdx.x; e < e_end; e += blockDim.x) {
    float v[KS];
#pragma unroll
    for (int r = 0; r < KS; ++r) v[r] = cluster.map_shared_rank(part, r)[e];
    float s = 0.f;
#pragma unroll
    for (int r = 0; r < KS; ++r) s += v[r];
    const int m = e / kSkCols, n = n_cta + e % kSkCols;
    if (m < M && n < N) {
      if (bias) s += load_scalar(bias, bias_dt, n);
      const int64_t o = (int64_t)m * ldy + n;
      if (accumulate) s += load_scalar(y, y_dt, o);
      store_scalar(y, y_dt, o, s);
    }
  }
  cluster.sync();  // no CTA leaves while another still reads its partial tile
}

template <int KS>
int launch_skinny(const __nv_bfloat16 *x, int64_t ldx, const __nv_bfloat16 *w, const void *bias, int bias_dt,
                  void *y, int y_dt, int64_t ldy, int accumulate, int M, int N, int K, int tiles,
                  cudaStream_t st) {
  if (KS > 8) {  // 16-CTA clusters are a non-portable size: opt in once
    static thread_local bool opted[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !opted[dev]) {
      const cudaError_t e =
          cudaFuncSetAttribute(skinny_gemm_kernel<KS>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      if (e != cudaSuccess)
        return set_error(DP_ERR_CUDA, std::string("dp_gemm_skinny: cluster size: ") + cudaGetErrorString(e));
      opted[dev] = true;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(KS, tiles, 1);
  cfg.blockDim = dim3(kSkWarps * 32, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = KS;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see pdl_wait
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, skinny_gemm_kernel<KS>, x, ldx, w, bias, bias_dt, y, y_dt, ldy,
                                           accumulate, M, N, K);
  if (e != cudaSuccess) return set_error(DP_ERR_CUDA, std::string("dp_gemm_skinny: ") + cudaGetErrorString(e));
  return check_launch("skinny_gemm_kernel");
}

}  // namespace
}  // namespace dp

extern "C" int dp_gemm_skinny(const void *x, int64_t ldx, const void *w, const void *bias, int bias_dtype, void *y,
                              int y_dtype, int64_t ldy, int accumulate, int M, int N, int K, void *stream) {
  using namespace dp;
  DP_REQUIRE(M >= 0 && N >= 0 && K >= 0, DP_ERR_INVALID_ARGUMENT, "dp_gemm_skinny: bad sizes");
  DP_REQUIRE(M <= 16, DP_ERR_UNSUPPORTED, "dp_gemm_skinny: M must be <= 16");
  DP_REQUIRE(valid_dtype(y_dtype) && (!bias || valid_dtype(bias_dtype)), DP_ERR_INVALID_ARGUMENT,
             "dp_gemm_skinny: bad dtype code");
  if (M == 0 || N == 0) return DP_OK;
  DP_REQUIRE(K % 32 == 0 && K > 0, DP_ERR_UNSUPPORTED, "dp_gemm_skinny: K must be a positive multiple of 32");
  DP_REQUIRE(x && w && y, DP_ERR_INVALID_ARGUMENT, "dp_gemm_skinny: null pointer");
  DP_REQUIRE(ldx >= K && ldy >= N, DP_ERR_INVALID_ARGUMENT, "dp_gemm_skinny: bad leading dimension");
  DP_REQUIRE(reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(w) % 16 == 0 && ldx % 8 == 0,
             DP_ERR_MISALIGNED, "dp_gemm_skinny: x and W must be 16-byte aligned, ldx a multiple of 8");
  // K split over a cluster of up to 16 CTAs: the most splits that divide K into 32-wide
  // steps and keep the grid within one wave
  const int tiles = (N + kSkCols - 1) / kSkCols;
  DP_REQUIRE(tiles <= 65535, DP_ERR_UNSUPPORTED, "dp_gemm_skinny: N too large");
  int ks = 16;
  while (ks > 1 && (K % (32 * ks) != 0 || (int64_t)tiles * ks > kSkWaveCtas)) ks >>= 1;
  const auto *xb = static_cast<const __nv_bfloat16 *>(x);
  const auto *wb = static_cast<const __nv_bfloat16 *>(w);
  cudaStream_t st = as_stream(stream);
  switch (ks) {
    case 16: return launch_skinny<16>(xb, ldx, wb, bias, bias_dtype, y, y_dtype, ldy, accumulate, M, N, K, tiles, st);
    case 8: return launch_skinny<8>(xb, ldx, wb, bias, bias_dtype, y, y_dtype, ldy, accumulate, M, N, K, tiles, st);
    case 4: return launch_skinny<4>(xb, ldx, wb, bias, bias_dtype, y, y_dtype, ldy, accumulate, M, N, K, tiles, st);
    case 2: return launch_skinny<2>(xb, ldx, wb, bias, bias_dtype, y, y_dtype, ldy, accumulate, M, N, K, tiles, st);
    default: return launch_skinny<1>(xb, ldx, wb, bias, bias_dtype, y, y_dtype, ldy, accumulate, M, N, K, tiles, st);
  }
}
