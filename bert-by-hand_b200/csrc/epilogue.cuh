// Epilogue output path shared by the tcgen05 GEMM kernels: bias (+ GELU) on 32 fp32
// accumulator columns, fp16 pack, and TMA stores through per-warp swizzled staging.
#pragma once

#include "common.cuh"
#include "internal.h"

namespace bbh {

constexpr int kMaxBiasCols = 2048;  // bias staged in shared memory when N <= this

// Output path of the epilogue: each warp owns 32 rows; a 64-column chunk of fp16 (32 words
// per row) is written to the warp's 4 KB staging buffer in the 128-byte-swizzle layout
// (16-byte piece c of row r at piece c ^ (r & 7), so the 32 lanes' row writes hit distinct
// banks), then lane 0 stores the 32 x 64 box with one TMA store. One proxy fence and one
// store per 64 columns; the buffer is rewritten only after the previous store has read it.
struct ChunkStore {
  uint8_t* buf;  // this warp's 4096 B (1024-byte aligned)
  const CUtensorMap* map;
  int lane;
  int issued = 0;

  __device__ __forceinline__ void put64(const uint32_t (&w)[32], int col0, int row0) {
    if (issued > 0) {
      if (lane == 0) bulk_wait_read<0>();
      __syncwarp();
    }
    uint8_t* rowp = buf + lane * 128;
    const int sw = lane & 7;
#pragma unroll
    for (int c = 0; c < 8; ++c)
      *reinterpret_cast<uint4*>(rowp + ((c ^ sw) << 4)) = make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
    fence_async_shared();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(map, buf, col0, row0);
      bulk_commit();
    }
    ++issued;
  }
  __device__ __forceinline__ void drain() {
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }
};

// Bias (+ GELU) on 32 accumulator columns, packed to 16 words of fp16 pairs.
// `bias` points at fp32 values in shared memory, or is null (then `gbias`, global fp16).
template <int EPI>
__device__ __forceinline__ void epi_pack32(const float* v, int col0, const float* bias, const __half* gbias, int N,
                                           uint32_t* w) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int col = col0 + j * 8;
    float b8[8];
    if (bias) {
      const float4 lo = *reinterpret_cast<const float4*>(bias + col);
      const float4 hi = *reinterpret_cast<const float4*>(bias + col + 4);
      b8[0] = lo.x, b8[1] = lo.y, b8[2] = lo.z, b8[3] = lo.w;
      b8[4] = hi.x, b8[5] = hi.y, b8[6] = hi.z, b8[7] = hi.w;
    } else if (gbias && col + 8 <= N) {
      unpack_half8(__ldg(reinterpret_cast<const uint4*>(gbias + col)), b8);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) b8[e] = 0.f;
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float y0 = v[j * 8 + 2 * e] + b8[2 * e];
      const float y1 = v[j * 8 + 2 * e + 1] + b8[2 * e + 1];
      w[j * 4 + e] = pack_half2(y0, y1);
      if constexpr (EPI == kEpiGelu) w[j * 4 + e] = gelu_half2(w[j * 4 + e]);
    }
  }
}

// One warp-level arrival (after all lanes' TMEM reads): lane 0 arrives for the warp.
__device__ __forceinline__ void warp_arrive(uint64_t* bar) {
  tc_fence_before();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

}  // namespace bbh
