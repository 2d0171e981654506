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

// Residual + bias + LayerNorm epilogue of one warp's 32-row x 64-column slice of an output
// row block whose 384 columns are split over two CTAs of a cluster (192 columns each,
// three 64-column warps per TMEM lane quadrant per CTA). Row statistics are combined in
// two levels: the three warps of a quadrant through shared memory (Chan et al.: for equal
// part sizes n, M2 = sum M2_i + n * sum (mean_i - mean)^2), then the two CTAs through
// distributed shared memory (st.async completing bytes on the partner's barrier).
// The warp's 32 x 64 residual slice is TMA-loaded into its staging buffer one tile ahead;
// the normalised output is written back over it in place and TMA-stored from there.
struct LnSlice {
  static constexpr int kParts = 3;  // warps per quadrant (64 columns each)
  uint8_t* buf;                 // this warp's 4096 B staging buffer (1024-aligned)
  const CUtensorMap* tmC;
  const CUtensorMap* tmR;
  uint64_t* res_bar;            // this warp's residual-landed barrier
  float* red;                   // [2 slots][2 stats][3 parts][128 rows]
  float2* xstat;                // [2 slots][128 rows] partner (mean, M2)
  uint64_t* xfull_bar;          // [2] partner statistics arrived
  uint32_t partner;             // cluster rank of the CTA with the other 192 columns
  const float* bias;            // [384] fp32 (shared memory)
  const float* gamma;
  const float* beta;
  float eps;
  int lane, quad, part, we;     // we = epilogue warp index (0 for the barrier's expect_tx)

  // lane 0: queue the residual slice of a tile (columns c0.., rows row0..)
  __device__ __forceinline__ void prefetch(int c0, int row0) const {
    if (lane == 0) {
      mbar_arrive_expect_tx(res_bar, 4096);
      tma_load_2d(buf, tmR, res_bar, c0, row0);
    }
  }

  // v = this lane's row, 64 fp32 accumulator columns starting at column c0. Returns false
  // when a wait ran out (abort). When has_next, the next tile's residual is queued as soon
  // as this tile's store has read the buffer.
  __device__ __forceinline__ bool finish(float (&v)[64], int iter, int c0, int row0, bool has_next, int nc0,
                                         int nrow0, volatile int* abort_flag, int* err) const {
    if (!mbar_wait(res_bar, iter & 1, abort_flag, err)) return false;
    uint8_t* rowp = buf + lane * 128;
    const int sw = lane & 7;
    uint4 res[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) res[j] = *reinterpret_cast<const uint4*>(rowp + ((j ^ sw) << 4));
    add32(v, bias + c0, &res[0]);
    add32(v + 32, bias + c0 + 32, &res[4]);
    // shifted sums (shift = this lane's first value) -> part mean and M2
    const float shift = v[0];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int j = 0; j < 64; ++j) {
      const float d = v[j] - shift;
      s1 += d;
      s2 += d * d;
    }
    // Two scratch slots alternate by tile, so one barrier per tile suffices: a warp can
    // rewrite a slot only after every part has passed the next tile's barrier.
    const int rloc = quad * 32 + lane;
    const int slot = iter & 1;
    float* rs = red + slot * (2 * kParts * 128);
    rs[part * 128 + rloc] = shift + s1 * (1.0f / 64);
    rs[kParts * 128 + part * 128 + rloc] = fmaxf(s2 - s1 * s1 * (1.0f / 64), 0.f);
    named_barrier(1 + quad, 32 * kParts);
    float mean_c = 0.f;
#pragma unroll
    for (int i = 0; i < kParts; ++i) mean_c += rs[i * 128 + rloc];
    mean_c *= 1.0f / kParts;
    float m2_c = 0.f;
#pragma unroll
    for (int i = 0; i < kParts; ++i) {
      const float d = rs[i * 128 + rloc] - mean_c;
      m2_c += rs[kParts * 128 + i * 128 + rloc] + d * d * 64;
    }
    // exchange with the partner CTA: part-0 lanes send their row's (mean, M2); one thread
    // per CTA posts the expected byte count on its own barrier. A slot is rewritten two
    // tiles later, after every part of this quadrant has passed the next tile's barrier,
    // so the receiver has read it by then.
    if (part == 0)
      st_async_f32x2(mapa_shared(smem_u32(&xstat[slot * 128 + rloc]), partner), mean_c, m2_c,
                     mapa_shared(smem_u32(&xfull_bar[slot]), partner));
    if (we == 0 && lane == 0) mbar_arrive_expect_tx(&xfull_bar[slot], 128 * 8);
    if (!mbar_wait_cluster(&xfull_bar[slot], (iter >> 1) & 1, abort_flag, err)) return false;
    const float2 ps = xstat[slot * 128 + rloc];
    const float dp = mean_c - ps.x;
    const float mean = 0.5f * (mean_c + ps.x);
    const float m2 = m2_c + ps.y + dp * dp * (0.5f * 192);
    const float rstd = rsqrtf(m2 * (1.0f / kHidden) + eps);
    // normalise, affine, write the row back over its residual, store the slice
    uint32_t w[32];
    pack32(v, c0, mean, rstd, w);
    pack32(v + 32, c0 + 32, mean, rstd, w + 16);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      *reinterpret_cast<uint4*>(rowp + ((j ^ sw) << 4)) = make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
    fence_async_shared();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(tmC, buf, c0, row0);
      bulk_commit();
      if (has_next) {
        bulk_wait_read<0>();
        mbar_arrive_expect_tx(res_bar, 4096);
        tma_load_2d(buf, tmR, res_bar, nc0, nrow0);
      }
    }
    return true;
  }

  __device__ __forceinline__ static void add32(float* v, const float* b, const uint4* res4) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float r8[8];
      unpack_half8(res4[j], r8);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[j * 8 + e] += b[j * 8 + e] + r8[e];
    }
  }

  __device__ __forceinline__ void pack32(const float* v, int col0, float mean, float rstd, uint32_t* w) const {
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 g = *reinterpret_cast<const float4*>(gamma + col0 + 4 * q);
      const float4 b = *reinterpret_cast<const float4*>(beta + col0 + 4 * q);
      const float* x = v + 4 * q;
      w[2 * q] = pack_half2((x[0] - mean) * rstd * g.x + b.x, (x[1] - mean) * rstd * g.y + b.y);
      w[2 * q + 1] = pack_half2((x[2] - mean) * rstd * g.z + b.z, (x[3] - mean) * rstd * g.w + b.w);
    }
  }
};

// One warp-level arrival (after all lanes' TMEM reads): lane 0 arrives for the warp.
__device__ __forceinline__ void warp_arrive(uint64_t* bar) {
  tc_fence_before();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

}  // namespace bbh
