// TMA tensor maps for the chunk inputs and outputs of the tensor-core kernels (core_tc.cu,
// core_pipe.cu, laplace_tc.cu): a (B, H, L, 64) tensor with element strides (s.b, s.h, s.t)
// and unit channel stride becomes a 4-d map with the channel innermost, then token, head
// and batch in the order of their strides, so one tiled copy (`cp.async.bulk.tensor.4d`, no
// multicast) moves one 64-token chunk of one (b, h).  Loads: tokens past L arrive as zeros.
// Stores (the float32 outputs of core_pipe.cu): tokens past L are not written.
#pragma once

#include <cuda.h>  // CUtensorMap and cuTensorMapEncodeTiled's types (called through the runtime)

#include "dp_common.cuh"

namespace dp {

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against the
// driver library); null if unavailable.
inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<EncodeTiledFn>(nullptr);
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// Dimension (1..3) of the map that holds token, head and batch.
struct ChunkMapDims {
  int8_t t, h, b;
};

// Encodes a 4-d map of a (B, H, L, C) tensor with unit channel stride: the channel
// innermost, then token, head and batch in the order of their strides, and a box of
// `box_channels` channels by 64 tokens.  Returns false if the driver rejects it (base not
// 16-byte aligned, a stride not a multiple of 16 bytes, ...).
inline bool encode_bhlc_map(CUtensorMap *m, ChunkMapDims *dims_out, const void *base, int B, int H, int L, int C,
                            const SeqStrides &s, CUtensorMapDataType dtype, int elem_bytes, int box_channels,
                            CUtensorMapSwizzle swizzle) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return false;
  const int64_t st[3] = {s.t, s.h, s.b};
  const int64_t ext[3] = {L, H, B};
  int ord[3] = {0, 1, 2};  // token, head, batch sorted by stride
  for (int i = 0; i < 3; ++i)
    for (int j = i + 1; j < 3; ++j)
      if (st[ord[j]] < st[ord[i]]) {
        const int tmp = ord[i];
        ord[i] = ord[j];
        ord[j] = tmp;
      }
  cuuint64_t dims[4] = {(cuuint64_t)C, 0, 0, 0};
  cuuint64_t strides[3];
  cuuint32_t box[4] = {(cuuint32_t)box_channels, 1, 1, 1};
  for (int i = 0; i < 3; ++i) {
    dims[i + 1] = (cuuint64_t)ext[ord[i]];
    strides[i] = (cuuint64_t)st[ord[i]] * elem_bytes;
    if (ord[i] == 0) {
      box[i + 1] = 64;
      dims_out->t = (int8_t)(i + 1);
    } else if (ord[i] == 1) {
      dims_out->h = (int8_t)(i + 1);
    } else {
      dims_out->b = (int8_t)(i + 1);
    }
  }
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return enc(m, dtype, 4, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
             CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Encodes the map of one bf16 input of 64 channels (base 16-byte aligned, strides
// multiples of 8 elements, L >= 64: the callers check these); returns false if the driver
// rejects it.  The box is `box_channels` channels (64: a whole token row; 8: one 16-byte
// column group, for loads straight into the core-matrix layout of an MMA operand) by 64
// tokens.  With swizzle128 (box_channels = 64 only) the 16-byte chunk c of a token row r
// lands at chunk c ^ (r % 8) of that row: threads that each read one row read
// conflict-free (the destination must be 1024-byte aligned).
inline bool encode_chunk_map(CUtensorMap *m, ChunkMapDims *dims_out, const void *base, int B, int H, int L,
                             const SeqStrides &s, int box_channels = 64, bool swizzle128 = false) {
  return encode_bhlc_map(m, dims_out, base, B, H, L, 64, s, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, box_channels,
                         swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE);
}

// The map of a float32 output of 64 channels for bulk tensor stores: a box of 32 channels
// (128 bytes) by 64 tokens with the 128-byte swizzle (16-byte chunk c of token row r at
// chunk c ^ (r % 8) in shared memory, 1024-byte aligned); tokens past L are not written.
inline bool encode_out_map(CUtensorMap *m, ChunkMapDims *dims_out, const float *base, int B, int H, int L,
                           const SeqStrides &s) {
  return encode_bhlc_map(m, dims_out, base, B, H, L, 64, s, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, 32,
                         CU_TENSOR_MAP_SWIZZLE_128B);
}

// One chunk (tokens t0 .. t0 + 63) of head h, batch b into 64 rows x 128 bytes of shared
// memory; completion counted in bytes on `bar` (8192 per call).  The channel coordinate is
// 0, so the innermost offset is 16-byte aligned.
__device__ __forceinline__ void tma_load_chunk(void *dst_smem, const CUtensorMap *m, ChunkMapDims d, int t0, int h,
                                               int b, uint64_t *bar) {
  const int c1 = d.t == 1 ? t0 : d.h == 1 ? h : b;
  const int c2 = d.t == 2 ? t0 : d.h == 2 ? h : b;
  const int c3 = d.t == 3 ? t0 : d.h == 3 ? h : b;
  const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(dst_smem));
  const uint32_t mb = static_cast<uint32_t>(__cvta_generic_to_shared(bar));
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
      "%5}], [%6];" ::"r"(dst),
      "l"(m), "r"(0), "r"(c1), "r"(c2), "r"(c3), "r"(mb)
      : "memory");
}

// Channels x0 .. x0 + 7 (x0 a multiple of 8: a 16-byte aligned start) of tokens t0 ..
// t0 + 63 of head h, batch b, through a map encoded with box_channels = 8: 64 rows of 16
// bytes, contiguous in shared memory; 1024 bytes counted on `bar`.
__device__ __forceinline__ void tma_load_colgroup(void *dst_smem, const CUtensorMap *m, ChunkMapDims d, int x0, int t0,
                                                  int h, int b, uint64_t *bar) {
  const int c1 = d.t == 1 ? t0 : d.h == 1 ? h : b;
  const int c2 = d.t == 2 ? t0 : d.h == 2 ? h : b;
  const int c3 = d.t == 3 ? t0 : d.h == 3 ? h : b;
  const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(dst_smem));
  const uint32_t mb = static_cast<uint32_t>(__cvta_generic_to_shared(bar));
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
      "%5}], [%6];" ::"r"(dst),
      "l"(m), "r"(x0), "r"(c1), "r"(c2), "r"(c3), "r"(mb)
      : "memory");
}

// Bulk tensor store of channels x0 .. x0 + 31 of tokens t0 .. t0 + 63 of head h, batch b
// from shared memory (a map of encode_out_map; x0 = 0 or 32), in the issuing thread's
// bulk-async group.
__device__ __forceinline__ void tma_store_chunk(const CUtensorMap *m, ChunkMapDims d, const void *src_smem, int x0,
                                                int t0, int h, int b) {
  const int c1 = d.t == 1 ? t0 : d.h == 1 ? h : b;
  const int c2 = d.t == 2 ? t0 : d.h == 2 ? h : b;
  const int c3 = d.t == 3 ? t0 : d.h == 3 ? h : b;
  const uint32_t src = static_cast<uint32_t>(__cvta_generic_to_shared(src_smem));
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%1, %2, %3, %4}], [%5];" ::"l"(m),
               "r"(x0), "r"(c1), "r"(c2), "r"(c3), "r"(src)
               : "memory");
}

__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// The issuing thread's bulk stores have finished reading their shared-memory source.
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

// The issuing thread's bulk stores are complete.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

}  // namespace dp
