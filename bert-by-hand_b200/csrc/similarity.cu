// The step after the path: cosine similarity of sentence pairs and its Spearman rank
// correlation with gold scores. Replaces the reference's evaluation in
// scripts/benchmark.py:54-61 (`sims = einsum("ij,ij->i", embs[a], embs[b])` on the unit
// embeddings, then scipy's spearmanr against the STS gold scores).
//   * bbh_pair_similarity (device): one warp per pair, 16-byte loads of both 384-wide fp16
//     rows (a warp reads each row as 768 contiguous bytes), fp32 products, shuffle sum.
//     HBM-bound: 1,536 B read + 8 B of indices + 4 B written per pair. An out-of-range
//     index gives NaN for that pair instead of a read out of bounds.
//   * bbh_spearman (host): Pearson correlation of the average ranks (ties share the mean
//     of their positions), in double precision.
#include "common.cuh"
#include "internal.h"
#include "../../include/bbh.h"

#include <algorithm>
#include <string>
#include <cmath>
#include <numeric>
#include <vector>

namespace {

constexpr int kSimWarps = 8;

__global__ void __launch_bounds__(kSimWarps * 32)
    pair_similarity_kernel(const __half* __restrict__ emb, int n, const int32_t* __restrict__ pairs, int m,
                           float* __restrict__ sims) {
  const int lane = threadIdx.x & 31;
  const int stride = gridDim.x * kSimWarps;
  for (int pi = blockIdx.x * kSimWarps + (threadIdx.x >> 5); pi < m; pi += stride) {
    const int a = pairs[2 * pi], b = pairs[2 * pi + 1];
    if (a < 0 || a >= n || b < 0 || b >= n) {
      if (lane == 0) sims[pi] = __int_as_float(0x7fc00000);
      continue;
    }
    // 384 fp16 = 48 pieces of 16 bytes: lanes 0..31 take pieces lane and lane + 32 (< 48)
    const uint4* ra = reinterpret_cast<const uint4*>(emb + static_cast<size_t>(a) * BBH_HIDDEN);
    const uint4* rb = reinterpret_cast<const uint4*>(emb + static_cast<size_t>(b) * BBH_HIDDEN);
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int piece = lane + 32 * k;
      if (piece < BBH_HIDDEN / 8) {
        float fa[8], fb[8];
        bbh::unpack_half8(__ldg(ra + piece), fa);
        bbh::unpack_half8(__ldg(rb + piece), fb);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc = fmaf(fa[e], fb[e], acc);
      }
    }
    acc = bbh::warp_sum(acc);
    if (lane == 0) sims[pi] = acc;
  }
}

// average ranks (1-based), ties share the mean of their positions
std::vector<double> average_ranks(const float* v, int n) {
  std::vector<int> idx(static_cast<size_t>(n));
  std::iota(idx.begin(), idx.end(), 0);
  std::stable_sort(idx.begin(), idx.end(), [&](int a, int b) { return v[a] < v[b]; });
  std::vector<double> r(static_cast<size_t>(n));
  for (int i = 0; i < n;) {
    int j = i;
    while (j + 1 < n && v[idx[j + 1]] == v[idx[i]]) ++j;
    const double avg = 0.5 * (i + j) + 1.0;
    for (int k = i; k <= j; ++k) r[size_t(idx[k])] = avg;
    i = j + 1;
  }
  return r;
}

}  // namespace

extern "C" {

int bbh_pair_similarity(const uint16_t* emb, int n, const int32_t* pairs, int m, float* sims, void* stream) {
  if (!emb || !pairs || !sims || n < 0 || m < 0 || (reinterpret_cast<uintptr_t>(emb) & 15))
    return bbh::internal_fail(BBH_ERR_ARG, "bbh_pair_similarity: bad arguments (emb must be 16-byte aligned)");
  if (m == 0) return BBH_OK;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int blocks = std::min((m + kSimWarps - 1) / kSimWarps, sms * 8);
  pair_similarity_kernel<<<blocks, kSimWarps * 32, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __half*>(emb), n, pairs, m, sims);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return bbh::internal_fail(BBH_ERR_CUDA, std::string("bbh_pair_similarity: ") + cudaGetErrorString(e));
  return BBH_OK;
}

int bbh_spearman(const float* x, const float* y, int n, double* rho) {
  if (!x || !y || !rho || n < 2) return bbh::internal_fail(BBH_ERR_ARG, "bbh_spearman: need n >= 2 pairs");
  for (int i = 0; i < n; ++i)
    if (std::isnan(x[i]) || std::isnan(y[i])) return bbh::internal_fail(BBH_ERR_ARG, "bbh_spearman: NaN input");
  const std::vector<double> rx = average_ranks(x, n), ry = average_ranks(y, n);
  const double mean = 0.5 * (n + 1);
  double sxy = 0, sxx = 0, syy = 0;
  for (int i = 0; i < n; ++i) {
    const double dx = rx[size_t(i)] - mean, dy = ry[size_t(i)] - mean;
    sxy += dx * dy;
    sxx += dx * dx;
    syy += dy * dy;
  }
  *rho = (sxx > 0 && syy > 0) ? sxy / std::sqrt(sxx * syy) : std::nan("");
  return BBH_OK;
}

}  // extern "C"
