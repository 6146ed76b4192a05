// Tensor-core (tcgen05) GEMM for the spectral Lerp FFN's two matrix products.
//
// Reference: LearnableSubstrateLerpFFN.forward (delta_phase/layers.py:119-141).  The FFN
// (csrc/ffn.cu) reduces to the DCT-II projection hdct = X Cdct^T and the folded combine
// y = z F; both are C (M x N) = A (M x K) B^T with A and B row-major along K (B = Cdct, or
// F^T), bf16 (kind::f16) or fp32 read as tf32 (kind::tf32) in, fp32 accumulation, and one
// of three epilogues:
//   * STORE_F32:  C -> fp32 (the DCT projection, read by the feature kernel);
//   * STORE_BF16: C -> bf16 (dp_ffn_fwd with bf16 activations);
//   * ADD_F32:    Y += C in fp32 (dp_ffn_fwd_residual: the block's residual add);
//   * SINCOS_BF16: cos C and sin C in bf16, to C's place and sin_off elements further (the
//     DCT branch's features, written straight into z: the projections never reach HBM).
//
// One persistent CTA per SM walks 256 x BN output tiles (BN = min(N, 256)); warp 0 streams
// 128-byte-wide K slabs (64 bf16 or 32 fp32) of A (256 rows) and B (BN rows) into a
// three-stage ring through TMA (128-byte swizzle, one tiled copy per operand and slab, no
// multicast); warp 1 issues the MMAs (two M = 128 halves sharing B, N = BN, one 32-byte K
// step each, both operands K-major from shared memory) into the two halves of tensor
// memory; warps 2-9 drain them (tcgen05.ld, one row per thread).  Tiles up to 128 wide
// have two accumulators (the epilogue of one tile runs under the MMAs of the next); 256-wide
// tiles one, the producer streaming the next tile's first slabs meanwhile.  A 256-row tile halves the B traffic per
// output of a 128-row one (the operands come from L2 at about 9 TB/s at full MMA rate).
// All waits are bounded: on expiry the kernel records DP_ERR_TIMEOUT, lets its copies and
// MMAs land and frees tensor memory.
#include <cstring>

#include "dp_common.cuh"
#include "tc_ptx.cuh"
#include "tmap.cuh"

namespace dp {

int *device_error_ptr();

namespace {

using namespace ptx;

constexpr int kBM = 256;        // rows of an output tile (two M = 128 MMA halves)
constexpr int kSlabBytes = 128;  // K slab per stage: one 128-byte swizzle row
constexpr int kStages = 3;
constexpr int kMaxBN = 256;
constexpr int kThreads = 320;   // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
constexpr int kEpiBase = 64;
constexpr uint64_t kTimeoutNs = 2000000000ull;
constexpr int A_STAGE = kBM * kSlabBytes;      // 32 KB
constexpr int B_STAGE = kMaxBN * kSlabBytes;   // 32 KB
constexpr int OFF_A = 0;
constexpr int OFF_B = OFF_A + kStages * A_STAGE;
constexpr int OFF_BAR = OFF_B + kStages * B_STAGE;
constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;  // + 1024: the operand base is rounded up to 1024 bytes

enum Epi : int { STORE_F32 = 0, STORE_BF16 = 1, ADD_F32 = 2, SINCOS_BF16 = 3 };

struct GemmArgs {
  void *c;          // output (fp32 or bf16), row-major with row stride ldc elements
  int64_t ldc;
  int64_t sin_off;  // SINCOS_BF16: elements from a cos output to its sin
  int M, N, K;
  int BN;           // tile width (a multiple of 32, <= 256, divides N)
  int nbuf;         // accumulators: 2 if BN <= 128, else 1
  int acc_cols;     // TMEM columns of one accumulator half (128 or 256)
  int n_tiles_n;    // N / BN
  int num_tiles;    // ceil(M / 256) * n_tiles_n
  int *err;
};

struct alignas(64) GemmMaps {
  CUtensorMap a, b;
};

struct GemmBars {
  uint64_t full[kStages], empty[kStages];
  uint64_t acc_full[2], acc_empty[2];
  uint32_t tmem_base;
  int fail;
};

// Shared-memory descriptor of a K-major operand in the 128-byte swizzle layout TMA writes:
// rows of 128 bytes (64 bf16), 8-row atoms of 1024 bytes (SBO), layout type 2.  A K step
// of 16 elements inside the atom advances the start address by 32 bytes.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1 << 16;                    // LBO (unused for swizzled K-major): 16 bytes
  d |= (uint64_t)(1024 >> 4) << 32;          // SBO: 8-row atom stride
  d |= (uint64_t)1 << 46;                    // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                    // SWIZZLE_128B
  return d;
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *m, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_u32(dst)),
      "l"(m), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// ------------------------------------------------------------------ TMA producer (warp 0)
template <typename T>
__device__ bool gemm_producer(const GemmArgs &g, const GemmMaps &maps, uint8_t *ops, GemmBars *bars) {
  constexpr int kBK = kSlabBytes / (int)sizeof(T);
  const int kslabs = g.K / kBK;
  const uint32_t bytes = (uint32_t)(A_STAGE + g.BN * kSlabBytes);
  int it = 0;
  for (int tile = blockIdx.x; tile < g.num_tiles; tile += gridDim.x) {
    const int m0 = (tile / g.n_tiles_n) * kBM, n0 = (tile % g.n_tiles_n) * g.BN;
    for (int ks = 0; ks < kslabs; ++ks, ++it) {
      const int s = it % kStages;
      if (it >= kStages && !mbar_wait(&bars->empty[s], (uint32_t)((it / kStages - 1) & 1), kTimeoutNs)) return false;
      mbar_arrive_expect_tx(&bars->full[s], bytes);
      tma_load_2d(ops + OFF_A + s * A_STAGE, &maps.a, ks * kBK, m0, &bars->full[s]);
      tma_load_2d(ops + OFF_B + s * B_STAGE, &maps.b, ks * kBK, n0, &bars->full[s]);
    }
  }
  // the copies in flight complete on `full`, which the MMA warp consumes; nothing else to wait for
  return true;
}

// ------------------------------------------------------------------ MMA issuer (warp 1)
// Accumulator b of a tile: rows 0..127 in TMEM columns (2 b) acc_cols .., rows 128..255 in
// (2 b + 1) acc_cols ....  Run by the whole warp: the waits by every lane, the MMAs and
// commits by one elected lane (warp-uniform operands issue faster than from a lane-0 branch).
template <typename T>
__device__ bool gemm_mma(const GemmArgs &g, uint8_t *ops, GemmBars *bars, uint32_t tmem) {
  constexpr bool kTf32 = sizeof(T) == 4;
  constexpr int kBK = kSlabBytes / (int)sizeof(T);
  const int kslabs = g.K / kBK;
  const uint32_t idesc = kTf32 ? idesc_tf32(128, g.BN, false, false) : idesc_bf16(128, g.BN, false, false);
  int it = 0, lt = 0;
  for (int tile = blockIdx.x; tile < g.num_tiles; tile += gridDim.x, ++lt) {
    const int buf = lt % g.nbuf;
    // the epilogue must have drained this accumulator (tile lt - nbuf)
    bool okw = lt < g.nbuf || mbar_wait(&bars->acc_empty[buf], (uint32_t)((lt / g.nbuf - 1) & 1), kTimeoutNs);
    if (!__all_sync(0xFFFFFFFFu, okw)) {
      if (lt > 0) mbar_wait(&bars->acc_full[(lt - 1) % g.nbuf], (uint32_t)(((lt - 1) / g.nbuf) & 1), kTimeoutNs);
      return false;
    }
    tc_fence_after();
    for (int ks = 0; ks < kslabs; ++ks, ++it) {
      const int s = it % kStages;
      okw = mbar_wait(&bars->full[s], (uint32_t)((it / kStages) & 1), kTimeoutNs);
      if (!__all_sync(0xFFFFFFFFu, okw)) {
        if (elect_one()) mma_commit(&bars->acc_full[buf]);  // let the issued MMAs land before returning
        __syncwarp();
        mbar_wait(&bars->acc_full[buf], (uint32_t)((lt / g.nbuf) & 1), kTimeoutNs);
        return false;
      }
      tc_fence_after();
      const uint32_t sa = smem_u32(ops + OFF_A + s * A_STAGE), sb = smem_u32(ops + OFF_B + s * B_STAGE);
      if (elect_one()) {
#pragma unroll
        for (int kk = 0; kk < kSlabBytes / 32; ++kk) {
          const uint64_t bd = desc_sw128(sb + kk * 32);
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            const uint64_t ad = desc_sw128(sa + half * (128 * kSlabBytes) + kk * 32);
            const uint32_t d = tmem + (uint32_t)((2 * buf + half) * g.acc_cols);
            if (kTf32)
              mma_tf32_ss(d, ad, bd, idesc, (ks | kk) != 0);
            else
              mma_f16_ss(d, ad, bd, idesc, (ks | kk) != 0);
          }
        }
        mma_commit(&bars->empty[s]);  // the slab's buffers are free once these MMAs have read them
      }
      __syncwarp();
    }
    if (elect_one()) mma_commit(&bars->acc_full[buf]);
    __syncwarp();
  }
  return true;
}

// ------------------------------------------------------------------ epilogue (warps 2-5)
// Warp w (2..9): lane quarter q = w % 4 and tile half hh = (w - 2) / 4; thread l owns row
// 128 hh + 32 q + l of every tile; 32 columns per tcgen05.ld, written as 16-byte stores.
// (Sixteen epilogue warps measured slower.)
template <int EPI>
__device__ bool gemm_epilogue(const GemmArgs &g, GemmBars *bars, uint32_t tmem) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, q = warp & 3, hh = (warp - 2) >> 2;
  const uint32_t lane_base = (uint32_t)(q * 32) << 16;
  int lt = 0;
  for (int tile = blockIdx.x; tile < g.num_tiles; tile += gridDim.x, ++lt) {
    const int buf = lt % g.nbuf;
    const int m = (tile / g.n_tiles_n) * kBM + 128 * hh + q * 32 + lane, n0 = (tile % g.n_tiles_n) * g.BN;
    if (!mbar_wait(&bars->acc_full[buf], (uint32_t)((lt / g.nbuf) & 1), kTimeoutNs)) return false;
    tc_fence_after();
    for (int j0 = 0; j0 < g.BN; j0 += 32) {
      float v[32];
      tmem_ld32_sync(tmem + lane_base + (uint32_t)((2 * buf + hh) * g.acc_cols + j0), v);
      if (m < g.M) {
        if (EPI == SINCOS_BF16) {
          __nv_bfloat16 *row = static_cast<__nv_bfloat16 *>(g.c) + (int64_t)m * g.ldc + n0 + j0;
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint32_t cw[4], sw[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              float s0, c0, s1, c1;
              sincos_2pi_fast(v[i + 2 * k], &s0, &c0);
              sincos_2pi_fast(v[i + 2 * k + 1], &s1, &c1);
              cw[k] = pack_bf16_rne(c0, c1);
              sw[k] = pack_bf16_rne(s0, s1);
            }
            *reinterpret_cast<uint4 *>(row + i) = make_uint4(cw[0], cw[1], cw[2], cw[3]);
            *reinterpret_cast<uint4 *>(row + g.sin_off + i) = make_uint4(sw[0], sw[1], sw[2], sw[3]);
          }
        } else if (EPI == STORE_BF16) {
          __nv_bfloat16 *row = static_cast<__nv_bfloat16 *>(g.c) + (int64_t)m * g.ldc + n0 + j0;
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 w;
            __nv_bfloat162 h0 = __floats2bfloat162_rn(v[i], v[i + 1]), h1 = __floats2bfloat162_rn(v[i + 2], v[i + 3]);
            __nv_bfloat162 h2 = __floats2bfloat162_rn(v[i + 4], v[i + 5]), h3 = __floats2bfloat162_rn(v[i + 6], v[i + 7]);
            w.x = *reinterpret_cast<uint32_t *>(&h0);
            w.y = *reinterpret_cast<uint32_t *>(&h1);
            w.z = *reinterpret_cast<uint32_t *>(&h2);
            w.w = *reinterpret_cast<uint32_t *>(&h3);
            *reinterpret_cast<uint4 *>(row + i) = w;
          }
        } else {
          float *row = static_cast<float *>(g.c) + (int64_t)m * g.ldc + n0 + j0;
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            float4 w = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
            if (EPI == ADD_F32) {
              const float4 o = *reinterpret_cast<const float4 *>(row + i);
              w.x += o.x;
              w.y += o.y;
              w.z += o.z;
              w.w += o.w;
            }
            *reinterpret_cast<float4 *>(row + i) = w;
          }
        }
      }
    }
    tc_fence_before();
    mbar_arrive(&bars->acc_empty[buf]);
  }
  return true;
}

template <typename T, int EPI>
__global__ void __launch_bounds__(kThreads, 1) gemm_tc_kernel(const __grid_constant__ GemmArgs g,
                                                              const __grid_constant__ GemmMaps maps) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned operand base (the 128-byte swizzle repeats every 1024 bytes)
  uint8_t *ops = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  GemmBars *bars = reinterpret_cast<GemmBars *>(ops + OFF_BAR);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&bars->full[i], 1);
      mbar_init(&bars->empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->acc_full[i], 1);
      mbar_init(&bars->acc_empty[i], kThreads - kEpiBase);
    }
    bars->fail = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, 2 * kMaxBN);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  bool ok = true;
  if (warp == 0) {
    if (lane == 0) ok = gemm_producer<T>(g, maps, ops, bars);
  } else if (warp == 1) {
    ok = gemm_mma<T>(g, ops, bars, tmem);
  } else {
    ok = gemm_epilogue<EPI>(g, bars, tmem);
  }
  if (!ok) atomicExch(&bars->fail, 1);
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && bars->fail) atomicCAS(g.err, 0, DP_ERR_TIMEOUT);
  if (warp == 1) tmem_dealloc(tmem, 2 * kMaxBN);
}

// 2-d map of a row-major matrix (rows x cols, row stride ld elements of es bytes), box of
// one 128-byte row segment x box_rows rows, 128-byte swizzle.
bool encode_2d_sw128(CUtensorMap *m, const void *base, int es, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)(ld * es)};
  const cuuint32_t box[2] = {(cuuint32_t)(kSlabBytes / es), (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, es == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
             const_cast<void *>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count() {
  static int n = [] {
    int dev = 0, v = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v > 0 ? v : 148;
  }();
  return n;
}

}  // namespace

// True if gemm_tc takes these sizes for elements of es bytes (2: bf16, 4: fp32 as tf32):
// N a multiple of 32 up to 256 or of 256 beyond, K a multiple of the 128-byte slab, A, B
// and their rows 16-byte aligned (TMA).
bool gemm_tc_supported(int es, const void *A, const void *B, int M, int N, int K, int64_t lda, int64_t ldb,
                       int bn_max) {
  const int bk = kSlabBytes / es;
  if (M <= 0 || N < 32 || K < bk || K % bk) return false;
  if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B)) & 15) return false;
  if (bn_max != 128 && bn_max != 256) return false;
  if (N > bn_max ? N % bn_max : N % 32) return false;
  return (lda * es) % 16 == 0 && (ldb * es) % 16 == 0;
}

// C (M x N) (epi) = A (M x K) B (N x K)^T, A and B row-major along K (strides lda, ldb
// elements, 16-byte aligned), bf16 (es = 2) or fp32 read as tf32 (es = 4).  epi: 0 store
// fp32, 1 store bf16, 2 add into fp32, 3 (bf16 only) cos to C and sin to C + sin_off.
// bn_max (128 or 256): the widest tile; 128 double-buffers the accumulator (for epilogues
// heavy enough to hide under the next tile's MMAs).
int gemm_tc(int es, const void *A, int64_t lda, const void *B, int64_t ldb, void *C, int64_t ldc, int M, int N, int K,
            int epi, cudaStream_t stream, int64_t sin_off, int bn_max) {
  if (!gemm_tc_supported(es, A, B, M, N, K, lda, ldb, bn_max))
    return set_error(DP_ERR_UNSUPPORTED, "gemm_tc: unsupported sizes or alignment");
  GemmArgs g;
  memset(&g, 0, sizeof(g));
  g.c = C;
  g.ldc = ldc;
  g.sin_off = sin_off;
  g.M = M;
  g.N = N;
  g.K = K;
  g.BN = N > bn_max ? bn_max : N;
  g.nbuf = g.BN <= 128 ? 2 : 1;
  g.acc_cols = g.nbuf == 2 ? 128 : 256;
  g.n_tiles_n = N / g.BN;
  g.num_tiles = ((M + kBM - 1) / kBM) * g.n_tiles_n;
  g.err = device_error_ptr();
  if (!g.err) return set_error(DP_ERR_CUDA, "gemm_tc: device error word unavailable");
  GemmMaps maps;
  memset(&maps, 0, sizeof(maps));
  if (!encode_2d_sw128(&maps.a, A, es, M, K, lda, kBM) || !encode_2d_sw128(&maps.b, B, es, N, K, ldb, g.BN))
    return set_error(DP_ERR_CUDA, "gemm_tc: tensor map encoding failed");
  void (*kern)(GemmArgs, GemmMaps);
  if (es == 2)
    kern = epi == STORE_F32    ? gemm_tc_kernel<__nv_bfloat16, STORE_F32>
           : epi == STORE_BF16 ? gemm_tc_kernel<__nv_bfloat16, STORE_BF16>
           : epi == ADD_F32    ? gemm_tc_kernel<__nv_bfloat16, ADD_F32>
                               : gemm_tc_kernel<__nv_bfloat16, SINCOS_BF16>;
  else
    kern = epi == ADD_F32 ? gemm_tc_kernel<float, ADD_F32> : gemm_tc_kernel<float, STORE_F32>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  if (e != cudaSuccess) return set_error(DP_ERR_CUDA, std::string("gemm_tc smem attr: ") + cudaGetErrorString(e));
  const int grid = g.num_tiles < sm_count() ? g.num_tiles : sm_count();
  kern<<<grid, kThreads, SMEM_BYTES, stream>>>(g, maps);
  return check_launch("gemm_tc_kernel");
}

}  // namespace dp
