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
// Embedding gather + LayerNorm (src/kernels/embedding.cu:8-31 + src/model/forward.cu:30).
// Token t of segment s sits at position t - start(s) (the reference's row % S, with S the
// padded length in padded mode). Also publishes the forward's segment table, per-token
// key/pool mask and {B, T, max_len} for the later kernels, and validates the inputs.
__global__ void __launch_bounds__(kRowThreads) embed_ln_kernel(EmbedParams p) {
  pdl_launch_dependents();
  pdl_wait();  // the previous forward's last kernels still read the buffers written here
  const int lane = threadIdx.x & 31;
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

  // Each warp takes `chunk` consecutive tokens at a time (2..8, enough to spread the
  // forward's tokens over all warps): lane l < chunk resolves token base + l (its segment
  // by binary search, position, ids, mask, validation) in parallel, then the warp gathers
  // and normalises the rows two at a time so both tokens' loads are in flight.
  const int chunk = min(8, max(2, ((p.total + warps - 1) / warps + 1) & ~1));
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
          if (__ldg(p.cu_seqlens + mid) <= t) lo = mid; else hi = mid;
        }
        pos = t - __ldg(p.cu_seqlens + lo);
      } else {
        pos = t % p.seq;
      }
      id = __ldg(p.ids + t);
      ty = p.types ? __ldg(p.types + t) : 0;
      if (id < 0 || id >= kVocab || ty < 0 || ty >= kTypes) set_dev_error(p.err, kDevBadToken);
      if (pos >= kMaxPos) set_dev_error(p.err, kDevBadPosition);
      p.ws_tokmask[t] = p.mask ? static_cast<uint8_t>(__ldg(p.mask + t) != 0) : uint8_t(1);
      id = (id < 0 || id >= kVocab) ? 0 : id;
      ty = (ty < 0 || ty >= kTypes) ? 0 : ty;
      pos = pos >= kMaxPos ? kMaxPos - 1 : pos;
      if (p.index_dump)  // the rows this token gathers, and whether it attends / is pooled
        *reinterpret_cast<int4*>(p.index_dump + 4 * static_cast<size_t>(t)) =
            make_int4(id, pos, ty, p.mask ? int(__ldg(p.mask + t) != 0) : 1);
    }
    const int n = min(chunk, p.total - base);
    for (int k = 0; k < n; k += 2) {
      const bool two = k + 1 < n;
      const int id0 = __shfl_sync(0xffffffffu, id, k), pos0 = __shfl_sync(0xffffffffu, pos, k);
      const int ty0 = __shfl_sync(0xffffffffu, ty, k);
      const int id1 = __shfl_sync(0xffffffffu, id, k + 1);
      const int pos1 = __shfl_sync(0xffffffffu, pos, k + 1);
      const int ty1 = __shfl_sync(0xffffffffu, ty, k + 1);
      float f0[12], f1[12], a[12], c[12];
      load_row12(p.word + static_cast<size_t>(id0) * kHidden, lane, f0);
      if (two) load_row12(p.word + static_cast<size_t>(id1) * kHidden, lane, f1);
      load_row12(p.pos + static_cast<size_t>(pos0) * kHidden, lane, a);
      load_row12(p.type + static_cast<size_t>(ty0) * kHidden, lane, c);
#pragma unroll
      for (int i = 0; i < 12; ++i) f0[i] += a[i] + c[i];
      warp_layernorm12(f0, p.gamma, p.beta, lane, p.eps);
      store_row12(p.out + static_cast<size_t>(base + k) * kHidden, lane, f0);
      if (two) {
        load_row12(p.pos + static_cast<size_t>(pos1) * kHidden, lane, a);
        load_row12(p.type + static_cast<size_t>(ty1) * kHidden, lane, c);
#pragma unroll
        for (int i = 0; i < 12; ++i) f1[i] += a[i] + c[i];
        warp_layernorm12(f1, p.gamma, p.beta, lane, p.eps);
        store_row12(p.out + static_cast<size_t>(base + k + 1) * kHidden, lane, f1);
      }
    }
  }
}

cudaError_t launch_embed_ln(const EmbedParams& p, int grid, cudaStream_t stream, bool pdl) {
  return launch_ex(embed_ln_kernel, dim3(grid), dim3(kRowThreads), 0, stream, pdl, 1, p);
}

// --------------------------------------------------------------------------------------
// Masked mean over each segment + L2 normalise (src/kernels/pooling.cu:8-32 and
// src/kernels/normalize.cu:10-33 fused). One 256-thread block per sentence: each warp
// sums a strided subset of the rows, partial sums meet in shared memory, warp 0
// normalises in fp32 and stores fp16 once. Empty segments give a zero vector, as
// (sum / max(count, 1)) / max(norm, 1e-12) does in the reference.
__global__ void __launch_bounds__(kRowThreads) pool_l2_kernel(PoolParams p) {
  __shared__ float part[kRowThreads / 32][kHidden];
  __shared__ int cnt[kRowThreads / 32];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  pdl_launch_dependents();
  pdl_wait();  // the hidden states come from the previous kernel
  const int batch = p.meta ? p.meta[0] : p.batch;
  for (int b = blockIdx.x; b < batch; b += gridDim.x) {
    const int start = p.cu[b];
    const int end = p.cu[b + 1];
    float acc[12];
#pragma unroll
    for (int i = 0; i < 12; ++i) acc[i] = 0.f;
    int n = 0;
    // each warp takes rows warp, warp + W, ... (W warps), four at a time so that their
    // loads are in flight together (the sentence's rows are independent until summed)
    constexpr int W = kRowThreads / 32;
    for (int t0 = start + warp; t0 < end; t0 += 4 * W) {
      uint2 u[4][3];
      bool use[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int t = t0 + r * W;
        use[r] = t < end && (!p.tokmask || p.tokmask[t]);
        if (use[r]) {
          const __half* row = p.hidden + static_cast<size_t>(t) * kHidden;
#pragma unroll
          for (int i = 0; i < 3; ++i) u[r][i] = __ldg(reinterpret_cast<const uint2*>(row + i * 128 + lane * 4));
        }
      }
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        if (!use[r]) continue;
#pragma unroll
        for (int i = 0; i < 3; ++i) {
          const __half2* hh = reinterpret_cast<const __half2*>(&u[r][i]);
          const float2 a = __half22float2(hh[0]);
          const float2 b = __half22float2(hh[1]);
          acc[i * 4 + 0] += a.x;
          acc[i * 4 + 1] += a.y;
          acc[i * 4 + 2] += b.x;
          acc[i * 4 + 3] += b.y;
        }
        ++n;
      }
    }
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) part[warp][i * 128 + lane * 4 + j] = acc[i * 4 + j];
    if (lane == 0) cnt[warp] = n;
    __syncthreads();
    if (warp == 0) {
      int count = 0;
#pragma unroll
      for (int w = 0; w < kRowThreads / 32; ++w) count += cnt[w];
      const float inv_cnt = 1.0f / static_cast<float>(count > 0 ? count : 1);
      float f[12];
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float s = 0.f;
#pragma unroll
          for (int w = 0; w < kRowThreads / 32; ++w) s += part[w][i * 128 + lane * 4 + j];
          s *= inv_cnt;
          f[i * 4 + j] = s;
          ss += s * s;
        }
      const float norm = sqrtf(warp_sum(ss));
      const float inv = 1.0f / fmaxf(norm, 1e-12f);
#pragma unroll
      for (int i = 0; i < 12; ++i) f[i] *= inv;
      store_row12(p.emb + static_cast<size_t>(b) * kHidden, lane, f);
    }
    __syncthreads();
  }
}

const void* embed_kernel_fn() { return reinterpret_cast<const void*>(embed_ln_kernel); }
const void* pool_kernel_fn() { return reinterpret_cast<const void*>(pool_l2_kernel); }

cudaError_t launch_pool_l2(const PoolParams& p, int grid, cudaStream_t stream, bool pdl) {
  return launch_ex(pool_l2_kernel, dim3(grid), dim3(kRowThreads), 0, stream, pdl, 1, p);
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
