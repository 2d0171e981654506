// Memory-bound row kernels: embedding gather + LayerNorm, masked mean-pool + L2
// normalise, and a standalone (residual) LayerNorm.
//
// Each 384-wide fp16 row is handled by one warp with 8-byte vector accesses (lane l owns
// columns 4l..4l+3, 128+4l.., 256+4l..), so a row is read once into registers and the
// statistics come from warp shuffles.
#include "common.cuh"
#include "internal.h"

namespace bbh {

constexpr int kRowThreads = 256;  // 8 warps

__device__ __forceinline__ void load_row12(const __half* row, int lane, float* f) {
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const uint2 u = __ldg(reinterpret_cast<const uint2*>(row + i * 128 + lane * 4));
    const __half2* h = reinterpret_cast<const __half2*>(&u);
    const float2 a = __half22float2(h[0]);
    const float2 b = __half22float2(h[1]);
    f[i * 4 + 0] = a.x;
    f[i * 4 + 1] = a.y;
    f[i * 4 + 2] = b.x;
    f[i * 4 + 3] = b.y;
  }
}

__device__ __forceinline__ void store_row12(__half* row, int lane, const float* f) {
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    uint2 u;
    u.x = pack_half2(f[i * 4 + 0], f[i * 4 + 1]);
    u.y = pack_half2(f[i * 4 + 2], f[i * 4 + 3]);
    *reinterpret_cast<uint2*>(row + i * 128 + lane * 4) = u;
  }
}

// In-register LayerNorm of one 384-wide row spread over a warp (two-pass statistics,
// like src/kernels/layernorm.cu:34-48), then affine.
__device__ __forceinline__ void warp_layernorm12(float* f, const __half* gamma, const __half* beta, int lane,
                                                 float eps) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 12; ++i) s += f[i];
  const float mean = warp_sum(s) * (1.0f / kHidden);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < 12; ++i) {
    const float d = f[i] - mean;
    q += d * d;
  }
  const float rstd = rsqrtf(warp_sum(q) * (1.0f / kHidden) + eps);
  float g[12], b[12];
  load_row12(gamma, lane, g);
  load_row12(beta, lane, b);
#pragma unroll
  for (int i = 0; i < 12; ++i) f[i] = (f[i] - mean) * rstd * g[i] + b[i];
}

// --------------------------------------------------------------------------------------
// 16-byte row access: a 384-wide fp16 row is 48 pieces of 16 bytes; a half-warp owns a row,
// lane h (0-15) the pieces h, h + 16 and h + 32 (24 values), so one load instruction of a
// warp moves two rows' 2 x 256 contiguous bytes and the row statistics need four shuffles.
__device__ __forceinline__ void ld_row24(const __half* row, int h, uint4 (&u)[3]) {
#pragma unroll
  for (int i = 0; i < 3; ++i) u[i] = __ldg(reinterpret_cast<const uint4*>(row) + i * 16 + h);
}

__device__ __forceinline__ void add_row24(const uint4 (&u)[3], float* f) {
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const __half2* hh = reinterpret_cast<const __half2*>(&u[i]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 x = __half22float2(hh[j]);
      f[i * 8 + 2 * j] += x.x;
      f[i * 8 + 2 * j + 1] += x.y;
    }
  }
}

__device__ __forceinline__ void st_row24(__half* row, int h, const float* f) {
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    uint4 u;
    u.x = pack_half2(f[i * 8 + 0], f[i * 8 + 1]);
    u.y = pack_half2(f[i * 8 + 2], f[i * 8 + 3]);
    u.z = pack_half2(f[i * 8 + 4], f[i * 8 + 5]);
    u.w = pack_half2(f[i * 8 + 6], f[i * 8 + 7]);
    reinterpret_cast<uint4*>(row)[i * 16 + h] = u;
  }
}

// sum over the 16 lanes of a half-warp
__device__ __forceinline__ float half_sum(float v) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// In-register LayerNorm of one row held by a half-warp (two-pass statistics, like
// src/kernels/layernorm.cu:34-48), then affine.
__device__ __forceinline__ void half_layernorm24(float* f, const __half* gamma, const __half* beta, int h,
                                                 float eps) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 24; ++i) s += f[i];
  const float mean = half_sum(s) * (1.0f / kHidden);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < 24; ++i) {
    const float d = f[i] - mean;
    q += d * d;
  }
  const float rstd = rsqrtf(half_sum(q) * (1.0f / kHidden) + eps);
  uint4 g[3], b[3];
  ld_row24(gamma, h, g);
  ld_row24(beta, h, b);
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const __half2* gg = reinterpret_cast<const __half2*>(&g[i]);
    const __half2* bb = reinterpret_cast<const __half2*>(&b[i]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 gf = __half22float2(gg[j]), bf = __half22float2(bb[j]);
      f[i * 8 + 2 * j] = (f[i * 8 + 2 * j] - mean) * rstd * gf.x + bf.x;
      f[i * 8 + 2 * j + 1] = (f[i * 8 + 2 * j + 1] - mean) * rstd * gf.y + bf.y;
    }
  }
}

// --------------------------------------------------------------------------------------
// Embedding gather + LayerNorm (src/kernels/embedding.cu:8-31 + src/model/forward.cu:30).
// Token t of segment s sits at position t - start(s) (the reference's row % S, with S the
// padded length in padded mode). Also publishes the forward's segment table, per-token
// key/pool mask and {B, T, max_len} for the later kernels, and validates the inputs.
constexpr int kSmemSegments = 4096;  // segment tables up to this size are searched in shared memory

__global__ void __launch_bounds__(kRowThreads) embed_ln_kernel(EmbedParams p) {
  __shared__ int s_cu[kSmemSegments + 1];
  pdl_launch_dependents();
  pdl_wait();  // the previous forward's last kernels still read the buffers written here
  const int lane = threadIdx.x & 31;
  const int half = lane >> 4;
  const int h = lane & 15;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  const int gwarp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const bool packed = p.cu_seqlens != nullptr;

  if (blockIdx.x == 0) {
    for (int b = threadIdx.x; b <= p.batch; b += blockDim.x) {
      int c = packed ? p.cu_seqlens[b] : b * p.seq;
      p.ws_cu[b] = c;
      if (packed && b > 0) {
        const int prev = p.cu_seqlens[b - 1];
        const int len = c - prev;
        if (len < 0 || len > p.max_len) set_dev_error(p.err, kDevBadSeqlens);
      }
    }
    if (threadIdx.x == 0) {
      if (packed && (p.cu_seqlens[0] != 0 || p.cu_seqlens[p.batch] != p.total)) set_dev_error(p.err, kDevBadSeqlens);
      p.ws_meta[0] = p.batch;
      p.ws_meta[1] = p.total;
      p.ws_meta[2] = p.max_len;
      p.ws_meta[3] = p.mask != nullptr ? 1 : 0;  // a key/pool mask is in effect
    }
  }

  // the segment offsets, once per block, for the per-token binary search
  const bool smem_cu = packed && p.batch <= kSmemSegments;
  if (smem_cu) {
    for (int b = threadIdx.x; b <= p.batch; b += blockDim.x) s_cu[b] = __ldg(p.cu_seqlens + b);
    __syncthreads();
  }
  const int* cu = smem_cu ? s_cu : p.cu_seqlens;

  // Each warp takes `chunk` consecutive tokens at a time (2..16, even, enough to spread the
  // forward's tokens over all warps): lane l < chunk resolves token base + l (its segment by
  // binary search, position, ids, mask, validation) in parallel; then the two half-warps
  // gather and normalise tokens base + 2k and base + 2k + 1, with the next pair's word rows
  // already being loaded while the current pair is normalised.
  const int chunk = min(16, max(2, ((p.total + warps - 1) / warps + 1) & ~1));
  for (int base = gwarp * chunk; base < p.total; base += warps * chunk) {
    const int t = base + lane;
    const bool valid = lane < chunk && t < p.total;
    int pos = 0, id = 0, ty = 0;
    if (valid) {
      if (packed) {
        // last segment whose start <= t (cu_seqlens is non-decreasing)
        int lo = 0, hi = p.batch;  // invariant: cu[lo] <= t < cu[hi]
        while (hi - lo > 1) {
          const int mid = (lo + hi) >> 1;
          if (cu[mid] <= t) lo = mid; else hi = mid;
        }
        pos = t - cu[lo];
      } else {
        pos = t % p.seq;
      }
      id = __ldg(p.ids + t);
      ty = p.types ? __ldg(p.types + t) : 0;
      if (id < 0 || id >= kVocab || ty < 0 || ty >= kTypes) set_dev_error(p.err, kDevBadToken);
      if (pos >= kMaxPos) set_dev_error(p.err, kDevBadPosition);
      const uint8_t m = p.mask ? static_cast<uint8_t>(__ldg(p.mask + t) != 0) : uint8_t(1);
      p.ws_tokmask[t] = m;
      id = (id < 0 || id >= kVocab) ? 0 : id;
      ty = (ty < 0 || ty >= kTypes) ? 0 : ty;
      pos = pos >= kMaxPos ? kMaxPos - 1 : pos;
      if (p.index_dump)  // the rows this token gathers, and whether it attends / is pooled
        *reinterpret_cast<int4*>(p.index_dump + 4 * static_cast<size_t>(t)) = make_int4(id, pos, ty, int(m));
    }
    const int n = min(chunk, p.total - base);
    // this half-warp's token of pair k is base + 2k + half (present when 2k + half < n)
    uint4 w[3];
    {
      const int idk = __shfl_sync(0xffffffffu, id, half);
      if (half < n) ld_row24(p.word + static_cast<size_t>(idk) * kHidden, h, w);
    }
    for (int k = 0; 2 * k < n; ++k) {
      const int src = 2 * k + half;
      const bool mine = src < n;
      const int posk = __shfl_sync(0xffffffffu, pos, src & 31);
      const int tyk = __shfl_sync(0xffffffffu, ty, src & 31);
      const int idn = __shfl_sync(0xffffffffu, id, (src + 2) & 31);
      uint4 wn[3], a[3], c[3];
      if (src + 2 < n) ld_row24(p.word + static_cast<size_t>(idn) * kHidden, h, wn);
      if (mine) {
        ld_row24(p.pos + static_cast<size_t>(posk) * kHidden, h, a);
        ld_row24(p.type + static_cast<size_t>(tyk) * kHidden, h, c);
        float f[24];
#pragma unroll
        for (int i = 0; i < 24; ++i) f[i] = 0.f;
        add_row24(w, f);
        add_row24(a, f);
        add_row24(c, f);
        half_layernorm24(f, p.gamma, p.beta, h, p.eps);
        st_row24(p.out + static_cast<size_t>(base + src) * kHidden, h, f);
      }
#pragma unroll
      for (int i = 0; i < 3; ++i) w[i] = wn[i];
    }
  }
}

cudaError_t launch_embed_ln(const EmbedParams& p, int grid, cudaStream_t stream, bool pdl) {
  return launch_ex(embed_ln_kernel, dim3(grid), dim3(kRowThreads), 0, stream, pdl, 1, p);
}

// --------------------------------------------------------------------------------------
// Masked mean over each segment + L2 normalise (src/kernels/pooling.cu:8-32 and
// src/kernels/normalize.cu:10-33 fused). One 128-thread block per sentence: its eight
// half-warps sum rows h, h + 8, ... of the sentence with 16-byte loads, four rows each in
// flight; the eight partial sums meet in shared memory, 48 threads finish one 16-byte
// piece of the mean each, and the L2 norm is reduced over the block. Empty segments give a
// zero vector, as (sum / max(count, 1)) / max(norm, 1e-12) does in the reference.
constexpr int kPoolThreads = 128;
__global__ void __launch_bounds__(kPoolThreads) pool_l2_kernel(PoolParams p) {
  constexpr int HW = kPoolThreads / 16;  // half-warps per block
  __shared__ __align__(16) float part[HW][kHidden];
  __shared__ int cnt[HW];
  __shared__ float sq[2];
  const int lane = threadIdx.x & 31;
  const int hw = threadIdx.x >> 4;
  const int h = lane & 15;
  pdl_launch_dependents();
  pdl_wait();  // the hidden states come from the previous kernel
  const int batch = p.meta ? p.meta[0] : p.batch;
  // packed forwards pool every token: no mask reads in front of the row loads
  const uint8_t* tokmask = (p.meta && p.meta[3] == 0) ? nullptr : p.tokmask;
  for (int b = blockIdx.x; b < batch; b += gridDim.x) {
    const int start = p.cu[b];
    const int end = p.cu[b + 1];
    float acc[24];
#pragma unroll
    for (int i = 0; i < 24; ++i) acc[i] = 0.f;
    int n = 0;
    for (int t0 = start + hw; t0 < end; t0 += 4 * HW) {
      uint4 u[4][3];
      bool use[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int t = t0 + r * HW;
        use[r] = t < end && (!tokmask || tokmask[t]);
        if (use[r]) ld_row24(p.hidden + static_cast<size_t>(t) * kHidden, h, u[r]);
      }
#pragma unroll
      for (int r = 0; r < 4; ++r)
        if (use[r]) {
          add_row24(u[r], acc);
          ++n;
        }
    }
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      float4* dst = reinterpret_cast<float4*>(&part[hw][(i * 16 + h) * 8]);
      dst[0] = make_float4(acc[i * 8 + 0], acc[i * 8 + 1], acc[i * 8 + 2], acc[i * 8 + 3]);
      dst[1] = make_float4(acc[i * 8 + 4], acc[i * 8 + 5], acc[i * 8 + 6], acc[i * 8 + 7]);
    }
    if (h == 0) cnt[hw] = n;
    __syncthreads();
    // thread j < 48 finishes columns 8j .. 8j+7
    const int j = threadIdx.x;
    float f[8];
    float ss = 0.f;
    if (j < 48) {
      int count = 0;
#pragma unroll
      for (int w = 0; w < HW; ++w) count += cnt[w];
      const float inv_cnt = 1.0f / static_cast<float>(count > 0 ? count : 1);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < HW; ++w) s += part[w][8 * j + e];
        f[e] = s * inv_cnt;
        ss += f[e] * f[e];
      }
    }
    if (threadIdx.x < 64) {
      ss = warp_sum(ss);
      if (lane == 0) sq[threadIdx.x >> 5] = ss;
    }
    __syncthreads();
    if (j < 48) {
      const float inv = 1.0f / fmaxf(sqrtf(sq[0] + sq[1]), 1e-12f);
      uint4 o;
      o.x = pack_half2(f[0] * inv, f[1] * inv);
      o.y = pack_half2(f[2] * inv, f[3] * inv);
      o.z = pack_half2(f[4] * inv, f[5] * inv);
      o.w = pack_half2(f[6] * inv, f[7] * inv);
      reinterpret_cast<uint4*>(p.emb + static_cast<size_t>(b) * kHidden)[j] = o;
    }
    __syncthreads();
  }
}

const void* embed_kernel_fn() { return reinterpret_cast<const void*>(embed_ln_kernel); }
const void* pool_kernel_fn() { return reinterpret_cast<const void*>(pool_l2_kernel); }

cudaError_t launch_pool_l2(const PoolParams& p, int grid, cudaStream_t stream, bool pdl) {
  return launch_ex(pool_l2_kernel, dim3(grid), dim3(kPoolThreads), 0, stream, pdl, 1, p);
}

// --------------------------------------------------------------------------------------
// Standalone LayerNorm of x (+ residual), D = 384: the reference's launch_layernorm
// (src/kernels/layernorm.cu:63-70). Not on the fused forward path (which folds the
// residual LayerNorm into the GEMM epilogue); exported for unit parity.
__global__ void __launch_bounds__(kRowThreads) layernorm_kernel(const __half* x, const __half* residual,
                                                                const __half* gamma, const __half* beta, __half* y,
                                                                int rows, float eps) {
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
    float f[12];
    load_row12(x + static_cast<size_t>(r) * kHidden, lane, f);
    if (residual) {
      float g[12];
      load_row12(residual + static_cast<size_t>(r) * kHidden, lane, g);
#pragma unroll
      for (int i = 0; i < 12; ++i) f[i] += g[i];
    }
    warp_layernorm12(f, gamma, beta, lane, eps);
    store_row12(y + static_cast<size_t>(r) * kHidden, lane, f);
  }
}

cudaError_t launch_layernorm(const __half* x, const __half* residual, const __half* gamma, const __half* beta,
                             __half* y, int rows, float eps, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  int grid = (rows + 7) / 8;
  if (grid > 148 * 16) grid = 148 * 16;
  layernorm_kernel<<<grid, kRowThreads, 0, stream>>>(x, residual, gamma, beta, y, rows, eps);
  return cudaGetLastError();
}

}  // namespace bbh
