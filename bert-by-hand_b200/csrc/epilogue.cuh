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

// ---------------------------------------------------------------- residual LayerNorm pieces
// Shared by every residual-LayerNorm epilogue (LnSlice below, gemm_ln.cu), so that all of
// them compute bit-identical results. The arithmetic runs on packed fp32 pairs (sm_100's
// f32x2 add / sub / mul / fma: two columns per instruction, each rounded as the scalar op).
__device__ __forceinline__ unsigned long long f2(float a, float b) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float2 f2_split(unsigned long long r) {
  float2 v;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(v.x), "=f"(v.y) : "l"(r));
  return v;
}
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ unsigned long long f2_sub(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ unsigned long long f2_mul(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ unsigned long long f2_fma(unsigned long long a, unsigned long long b,
                                                     unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// x = accumulator + (bias + residual) for 8 columns: acc[8] fp32, bias[8] fp32 (16-byte
// aligned), res = 8 fp16 values; x as four packed pairs.
__device__ __forceinline__ void ln_x8(const float* acc, const float* bias, uint4 res, unsigned long long (&x)[4]) {
  const __half2* h = reinterpret_cast<const __half2*>(&res);
  const float4 b0 = *reinterpret_cast<const float4*>(bias);
  const float4 b1 = *reinterpret_cast<const float4*>(bias + 4);
  const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 r = __half22float2(h[e]);
    x[e] = f2_add(f2(acc[2 * e], acc[2 * e + 1]), f2_add(f2(bb[2 * e], bb[2 * e + 1]), f2(r.x, r.y)));
  }
}

// x = accumulator + (bias + residual) over 64 columns of one row, in place (v[64] holds the
// fp32 accumulator on entry and x on return; bias[64], res[8] as for ln_x8), and the mean
// and M2 (sum of squared deviations) of x, from sums shifted by the first x; even and odd
// columns accumulate in the two halves of packed pairs and are added at the end.
__device__ __forceinline__ void ln_stats64(float* v, const float* bias, const uint4* res, float& mean, float& m2) {
  unsigned long long s1 = f2(0.f, 0.f), s2 = f2(0.f, 0.f), sh = 0;
  float shift = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    unsigned long long x[4];
    ln_x8(v + 8 * j, bias + 8 * j, res[j], x);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if (j == 0 && e == 0) {
        shift = f2_split(x[0]).x;
        sh = f2(shift, shift);
      }
      const unsigned long long d = f2_sub(x[e], sh);
      s1 = f2_add(s1, d);
      s2 = f2_fma(d, d, s2);
      const float2 xf = f2_split(x[e]);
      v[8 * j + 2 * e] = xf.x;
      v[8 * j + 2 * e + 1] = xf.y;
    }
  }
  const float2 a = f2_split(s1), b = f2_split(s2);
  const float t1 = a.x + a.y, t2 = b.x + b.y;
  mean = shift + t1 * (1.0f / 64);
  m2 = fmaxf(t2 - t1 * t1 * (1.0f / 64), 0.f);
}

// (x - mean) * rstd * gamma + beta for 64 columns of x starting at column col, packed fp16
// into 8 16-byte pieces.
__device__ __forceinline__ void ln_norm64(const float* x, const float* gamma, const float* beta, int col,
                                          unsigned long long mean2, unsigned long long rstd2, uint4* out) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float4 g0 = *reinterpret_cast<const float4*>(gamma + col + 8 * j);
    const float4 g1 = *reinterpret_cast<const float4*>(gamma + col + 8 * j + 4);
    const float4 c0 = *reinterpret_cast<const float4*>(beta + col + 8 * j);
    const float4 c1 = *reinterpret_cast<const float4*>(beta + col + 8 * j + 4);
    const float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
    const float cc[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const unsigned long long xe = f2(x[8 * j + 2 * e], x[8 * j + 2 * e + 1]);
      const unsigned long long t = f2_mul(f2_sub(xe, mean2), rstd2);
      const float2 o = f2_split(f2_fma(t, f2(gg[2 * e], gg[2 * e + 1]), f2(cc[2 * e], cc[2 * e + 1])));
      w[e] = pack_half2(o.x, o.y);
    }
    out[j] = make_uint4(w[0], w[1], w[2], w[3]);
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
    float pmean, pm2;
    ln_stats64(v, bias + c0, res, pmean, pm2);
    // Two scratch slots alternate by tile, so one barrier per tile suffices: a warp can
    // rewrite a slot only after every part has passed the next tile's barrier.
    const int rloc = quad * 32 + lane;
    const int slot = iter & 1;
    float* rs = red + slot * (2 * kParts * 128);
    rs[part * 128 + rloc] = pmean;
    rs[kParts * 128 + part * 128 + rloc] = pm2;
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
    uint4 y[8];
    ln_norm64(v, gamma, beta, c0, f2(mean, mean), f2(rstd, rstd), y);
#pragma unroll
    for (int j = 0; j < 8; ++j) *reinterpret_cast<uint4*>(rowp + ((j ^ sw) << 4)) = y[j];
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
};

// One warp-level arrival (after all lanes' TMEM reads): lane 0 arrives for the warp.
__device__ __forceinline__ void warp_arrive(uint64_t* bar) {
  tc_fence_before();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

}  // namespace bbh
