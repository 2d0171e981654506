// CTA-pair (cta_group::2) tcgen05 GEMM with the residual LayerNorm epilogue over whole
// 384-wide rows, for the encoder's two N = 384 projections:
//   C[rows, 384] = LayerNorm(A[rows, K] . W[384, K]^T + bias + R) * gamma + beta
// i.e. the attention output projection (K = 384) and the second FFN layer (K = 1536), each
// followed by the reference's residual LayerNorm (src/kernels/matmul.cu:94-186, then
// src/kernels/layernorm.cu:17-59, called at src/model/encoder.cu:47-50 and :61-64).
//
// One SM pair owns a 256 x 384 output tile: the even CTA issues two M = 256, N = 192 MMAs per
// K step (columns 0-191 and 192-383) whose B operands are 96-row halves of W held by the two
// CTAs, so each CTA holds 128 accumulator rows x all 384 columns in TMEM. A row's
// statistics then never leave the CTA: each A tile is loaded once per pair and no
// distributed-shared-memory exchange is needed (a layout of two pairs per 4-CTA cluster,
// 192 columns each, loads every A tile twice and exchanges statistics between the pairs).
// The price is one TMEM accumulator (384 of 512 columns): the epilogue of tile i and the
// MMAs of tile i + 1 do not overlap, while the producer already streams tile i + 1's
// operands into the ring.
//
// Epilogue: 8 warps, 2 per TMEM lane quadrant, 192 columns (three 64-column chunks) each,
// one row per thread. Each warp's residual chunks are TMA-loaded into three 4 KB staging
// buffers during the MMAs. Pass 1 reads each chunk of the accumulator, adds bias and
// residual, takes the chunk's shifted sums and writes the fp32 sum back over the
// accumulator in TMEM; the two warps of a quadrant combine their statistics through shared
// memory; pass 2 reads the sums back, normalises, writes fp16 over the residual in the
// staging buffers and TMA-stores them; the next tile's residual is requested once the
// stores have read the buffers. The arithmetic (ln_stats64 / ln_norm64 in epilogue.cuh,
// three 64-column parts combined per 192 columns, then the two 192-column halves) is the
// one LnSlice uses in the one-SM kernel, so both give bit-identical results.
//
// Every mbarrier wait is bounded (mbar_wait*); no TMA multicast anywhere.
#include "common.cuh"
#include "epilogue.cuh"
#include "internal.h"
#include "../../include/bbh.h"

namespace bbh {

// Optional wait-time accounting for tuning (compiled only with -DBBH_GEMM_TRACE), summed
// over CTAs in clock64 cycles: [0] MMA thread waiting for the accumulator to be released,
// [1] MMA thread waiting for operands, [2] epilogue waiting for a finished accumulator,
// [3] epilogue waiting for residual chunks, [4] epilogue pass 1, [5] epilogue statistics
// exchange, [6] epilogue pass 2, [7] tiles (epilogue warp 2), [8] kernel span of warps 1 and
// 2 in globaltimer ns.
#ifdef BBH_GEMM_TRACE
__device__ unsigned long long g_ln_trace[16];
#define LN_T0() const long long tt_ = clock64()
#define LN_ACC(slot) trace[slot] += clock64() - tt_
#else
#define LN_T0()
#define LN_ACC(slot)
#endif

struct LnPairCfg {
  static constexpr int BM = 128;                         // accumulator rows per CTA (256 per pair)
  static constexpr int BK = 64;                          // one 128-byte swizzle row of fp16
  static constexpr int NH = 192;                         // columns per MMA; two cover the row
  static constexpr int B_ROWS = NH / 2;                  // W rows per CTA per MMA
  static constexpr int A_BYTES = BM * BK * 2;            // 16 KB
  static constexpr int B_BYTES = 2 * B_ROWS * BK * 2;    // 24 KB: two 96-row boxes
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;  // 40 KB
  static constexpr int EPI_WARPS = 8;                    // 2 per TMEM lane quadrant
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int CHUNKS = 3;                       // 64-column chunks per warp
  static constexpr int STAGING_BYTES = EPI_WARPS * CHUNKS * 4096;
  static constexpr int AUX_BYTES = 1024 /*barriers*/ + 3 * 4 * kHidden /*bias, gamma, beta*/ +
                                   2 * 2 * 128 * 8 /*quadrant statistics, 2 slots x 2 halves*/;
  static constexpr int RING_BYTES = 227 * 1024 - 1024 - STAGING_BYTES - AUX_BYTES;
  static constexpr int STAGES = RING_BYTES / STAGE_BYTES;
  static constexpr int TMEM_COLS = 512;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + STAGING_BYTES + AUX_BYTES;
  static_assert(STAGES >= 3, "operand ring too shallow");
  static_assert(SMEM <= 227 * 1024, "shared memory over the per-CTA limit");
  static_assert(2 * NH == kHidden && 2 * NH <= TMEM_COLS, "one 384-column accumulator");
};

__global__ void __launch_bounds__(LnPairCfg::THREADS, 1)
    gemm_ln_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmR,
                        GemmParams p) {
  using Cfg = LnPairCfg;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int CH = Cfg::CHUNKS;

  extern __shared__ uint8_t smem_raw[];
  // the same 1024-aligned offsets in both CTAs: the pair MMA reads both at one address
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;  // per stage: W rows for columns 0-191, then 192-383
  uint8_t* s_stage = smem + STAGES * Cfg::STAGE_BYTES;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(s_stage + Cfg::STAGING_BYTES);  // used in the even CTA
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* accf_bar = empty_bar + STAGES;   // [1]
  uint64_t* acce_bar = accf_bar + 1;         // [1] used in the even CTA
  uint64_t* res_bar = acce_bar + 1;          // [EPI_WARPS][CHUNKS] residual chunk landed
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(res_bar + Cfg::EPI_WARPS * CH);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* s_bias = reinterpret_cast<float*>(s_stage + Cfg::STAGING_BYTES + 1024);  // [384]
  float* s_gamma = s_bias + kHidden;                                               // [384]
  float* s_beta = s_gamma + kHidden;                                               // [384]
  float2* xs = reinterpret_cast<float2*>(s_beta + kHidden);  // [2 slots][2 halves][128 rows] (mean, M2)

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();
  const uint32_t lead_rank = crank & ~1u;
  const bool leader = crank == lead_rank;
  const int half = static_cast<int>(crank & 1);  // which 128 rows of the pair tile
#ifdef BBH_GEMM_TRACE
  long long trace[10] = {};
  const unsigned long long g_start = globaltimer();
#endif

  pdl_launch_dependents();
  const int k_blocks = (p.K + Cfg::BK - 1) / Cfg::BK;
  const int first_tile = static_cast<int>(blockIdx.x) / 2;
  const int tile_step = static_cast<int>(gridDim.x) / 2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);   // the even CTA's producer arrival (+ both CTAs' bytes)
      mbar_init(&empty_bar[s], 1);  // one commit from the MMA thread
    }
    mbar_init(&accf_bar[0], 1);
    mbar_init(&acce_bar[0], 2 * Cfg::EPI_WARPS);  // every epilogue warp of both CTAs
    for (int i = 0; i < Cfg::EPI_WARPS * CH; ++i) mbar_init(&res_bar[i], 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
    tma_prefetch_desc(&tmR);
  }
  if (warp == 1) tmem_alloc_pair(tmem_holder, Cfg::TMEM_COLS);
  for (int i = threadIdx.x; i < kHidden; i += blockDim.x) {
    s_bias[i] = p.bias ? __half2float(p.bias[i]) : 0.f;
    s_gamma[i] = __half2float(p.gamma[i]);
    s_beta[i] = __half2float(p.beta[i]);
  }
  pdl_wait();
  const int rows = p.rows_dev ? *p.rows_dev : p.rows;
  const int num_tiles = (rows + 2 * Cfg::BM - 1) / (2 * Cfg::BM);
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  auto tile_m0 = [&](int t) { return t * (2 * Cfg::BM) + half * Cfg::BM; };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      const uint32_t full0 = mapa_shared(smem_u32(full_bar), lead_rank);
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = first_tile; tile < num_tiles && !*abort_flag; tile += tile_step) {
        const int m0 = tile_m0(tile);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag, p.err)) break;
          if (leader) mbar_arrive_expect_tx(&full_bar[stage], 2 * Cfg::STAGE_BYTES);
          const uint32_t fb = full0 + stage * 8;
          uint8_t* b = sB + stage * Cfg::B_BYTES;
          tma_load_2d_pair(sA + stage * Cfg::A_BYTES, &tmA, fb, kb * Cfg::BK, m0);
          tma_load_2d_pair(b, &tmB, fb, kb * Cfg::BK, half * Cfg::B_ROWS);
          tma_load_2d_pair(b + Cfg::B_BYTES / 2, &tmB, fb, kb * Cfg::BK, Cfg::NH + half * Cfg::B_ROWS);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    if (leader && lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(2 * Cfg::BM, Cfg::NH);
      const uint32_t empty_peer = mapa_shared(smem_u32(empty_bar), crank + 1);
      const uint32_t accf_peer = mapa_shared(smem_u32(accf_bar), crank + 1);
      int stage = 0;
      uint32_t phase = 0, acc_phase = 0;
      for (int tile = first_tile; tile < num_tiles && !*abort_flag; tile += tile_step) {
        {
          LN_T0();
          if (!mbar_wait(&acce_bar[0], acc_phase ^ 1, abort_flag, p.err)) break;
          LN_ACC(0);
        }
        tc_fence_after();
        bool ok = true;
        for (int kb = 0; kb < k_blocks; ++kb) {
          LN_T0();
          if (!mbar_wait(&full_bar[stage], phase, abort_flag, p.err)) {
            ok = false;
            break;
          }
          LN_ACC(1);
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * Cfg::A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * Cfg::B_BYTES);
#pragma unroll
          for (int k = 0; k < Cfg::BK / 16; ++k) {
            const uint32_t acc = (kb | k) != 0 ? 1u : 0u;
            const uint64_t ad = sw128_kmajor_desc(a_addr + k * 32);
            tc_mma_f16_pair(tmem_base, ad, sw128_kmajor_desc(b_addr + k * 32), idesc, acc);
            tc_mma_f16_pair(tmem_base + Cfg::NH, ad, sw128_kmajor_desc(b_addr + Cfg::B_BYTES / 2 + k * 32), idesc,
                            acc);
          }
          // the slot is free in both CTAs once these MMAs have read it
          tc_commit_pair(smem_u32(&empty_bar[stage]));
          tc_commit_pair(empty_peer + stage * 8);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit_pair(smem_u32(&accf_bar[0]));
        tc_commit_pair(accf_peer);
        acc_phase ^= 1;
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int we = warp - 2;          // epilogue warp index
    const int quad = warp & 3;        // TMEM lane quadrant this warp may access
    const int hc = we >> 2;           // which 192 columns of the row (0 or 1)
    const int rloc = quad * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t acce0 = mapa_shared(smem_u32(acce_bar), lead_rank);
    const int col_base = hc * Cfg::NH;
    uint8_t* buf0 = s_stage + we * CH * 4096;  // the warp's three 32 x 64 chunk buffers
    uint64_t* rb = res_bar + we * CH;
    const int sw = lane & 7;
    auto request_residual = [&](int tile) {
      if (lane == 0)
        for (int j = 0; j < CH; ++j) {
          mbar_arrive_expect_tx(&rb[j], 4096);
          tma_load_2d(buf0 + j * 4096, &tmR, &rb[j], col_base + j * 64, tile_m0(tile) + quad * 32);
        }
    };
    if (first_tile < num_tiles) request_residual(first_tile);
    int iter = 0;
    for (int tile = first_tile; tile < num_tiles; tile += tile_step, ++iter) {
      const int row0 = tile_m0(tile) + quad * 32;
      {
        LN_T0();
        if (!mbar_wait(&accf_bar[0], iter & 1, abort_flag, p.err)) break;
        LN_ACC(2);
      }
#ifdef BBH_GEMM_TRACE
      const long long tp1 = clock64();
#endif
      tc_fence_after();
      const uint32_t tacc = tmem_base + lane_off + col_base;
      // pass 1: x = accumulator + bias + residual per chunk, its statistics, x back to TMEM
      float pmean[CH], pm2[CH];
      bool ok = true;
#pragma unroll
      for (int j = 0; j < CH; ++j) {
        float v[64];
        tmem_ld64(tacc + j * 64, tacc + j * 64 + 32, v);
        {
          LN_T0();
          if (!mbar_wait(&rb[j], iter & 1, abort_flag, p.err)) {
            ok = false;
            break;
          }
          LN_ACC(3);
        }
        const uint8_t* rowp = buf0 + j * 4096 + lane * 128;
        uint4 res[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) res[q] = *reinterpret_cast<const uint4*>(rowp + ((q ^ sw) << 4));
        ln_stats64(v, s_bias + col_base + j * 64, res, pmean[j], pm2[j]);
        tmem_st32(tacc + j * 64, *reinterpret_cast<const float(*)[32]>(v));
        tmem_st32(tacc + j * 64 + 32, *reinterpret_cast<const float(*)[32]>(v + 32));
      }
      if (!ok) break;
#ifdef BBH_GEMM_TRACE
      trace[4] += clock64() - tp1;
      const long long tx = clock64();
#endif
      float mean_c = 0.f;
#pragma unroll
      for (int j = 0; j < CH; ++j) mean_c += pmean[j];
      mean_c *= 1.0f / CH;
      float m2_c = 0.f;
#pragma unroll
      for (int j = 0; j < CH; ++j) {
        const float d = pmean[j] - mean_c;
        m2_c += pm2[j] + d * d * 64;
      }
      // the other 192 columns of this row belong to the partner warp of the quadrant
      const int slot = iter & 1;
      xs[(slot * 2 + hc) * 128 + rloc] = make_float2(mean_c, m2_c);
      named_barrier(1 + quad, 64);
      const float2 ps = xs[(slot * 2 + (hc ^ 1)) * 128 + rloc];
      const float dp = mean_c - ps.x;
      const float mean = 0.5f * (mean_c + ps.x);
      const float m2 = m2_c + ps.y + dp * dp * (0.5f * 192);
      const float rstd = rsqrtf(m2 * (1.0f / kHidden) + p.eps);
      const unsigned long long mean2 = f2(mean, mean), rstd2 = f2(rstd, rstd);
#ifdef BBH_GEMM_TRACE
      trace[5] += clock64() - tx;
      const long long tp2 = clock64();
#endif
      // pass 2: x back from TMEM, normalised, affine, fp16 over the residual, TMA store
#pragma unroll 1
      for (int j = 0; j < CH; ++j) {
        const int c0 = col_base + j * 64;
        float v[64];
        tmem_ld64(tacc + j * 64, tacc + j * 64 + 32, v);
        if (j == CH - 1) {
          // accumulator fully read by this warp: release it to the even CTA's MMA thread
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(acce0);
        }
        uint4 out[8];
        ln_norm64(v, s_gamma, s_beta, c0, mean2, rstd2, out);
        uint8_t* rowp = buf0 + j * 4096 + lane * 128;
#pragma unroll
        for (int q = 0; q < 8; ++q) *reinterpret_cast<uint4*>(rowp + ((q ^ sw) << 4)) = out[q];
        fence_async_shared();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmC, buf0 + j * 4096, c0, row0);
          bulk_commit();
        }
      }
#ifdef BBH_GEMM_TRACE
      trace[6] += clock64() - tp2;
      trace[7] += 1;
#endif
      // the next tile's residual goes into the buffers once the stores have read them
      const int nt = tile + tile_step;
      if (nt < num_tiles) {
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
        request_residual(nt);
      }
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

#ifdef BBH_GEMM_TRACE
  trace[8] = static_cast<long long>(globaltimer() - g_start);
  if (lane == 0 && (warp == 1 || warp == 2))
    for (int i = 0; i < 10; ++i) atomicAdd(&g_ln_trace[i], static_cast<unsigned long long>(trace[i]));
#endif
  tc_fence_before();
  __syncthreads();
  if (*abort_flag && warp == 0 && lane == 0) {
    // Let in-flight TMA copies land before the CTA's shared memory is released.
    const unsigned long long t0 = globaltimer();
    while (globaltimer() - t0 < 1000000ull) {
    }
  }
  __syncthreads();
  cluster_sync_all();  // the other CTA no longer reads or signals this CTA's memory
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
}

cudaError_t launch_gemm_ln_pair(const GemmPlan& plan, cudaStream_t stream, bool pdl) {
  using Cfg = LnPairCfg;
  if (!plan.p.residual || !plan.p.gamma || !plan.p.beta || plan.p.N != kHidden) return cudaErrorInvalidValue;
  static bool attr_set[64] = {};
  static int max_clusters[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  auto kern = gemm_ln_pair_kernel;
  if (dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * 74);
    cfg.blockDim = dim3(Cfg::THREADS);
    cfg.dynamicSmemBytes = Cfg::SMEM;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
    if (e != cudaSuccess || n <= 0) n = 64;
    max_clusters[dev] = n;
    attr_set[dev] = true;
  }
  const int tiles_cap = (plan.rows_cap + 255) / 256;
  int nclusters = dev < 64 ? max_clusters[dev] : 64;
  if (nclusters > tiles_cap) nclusters = tiles_cap;
  return launch_ex(kern, dim3(2 * nclusters), dim3(Cfg::THREADS), Cfg::SMEM, stream, pdl, 2, plan.tmA, plan.tmB2,
                   plan.tmC, plan.tmR, plan.p);
}

}  // namespace bbh

#ifdef BBH_GEMM_TRACE
extern "C" __attribute__((visibility("default"))) int bbh_ln_trace(unsigned long long* out, int reset) {
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  if (cudaMemcpyFromSymbol(out, bbh::g_ln_trace, sizeof(unsigned long long) * 16) != cudaSuccess) return -1;
  if (reset) {
    unsigned long long z[16] = {};
    cudaMemcpyToSymbol(bbh::g_ln_trace, z, sizeof(z));
  }
  return 0;
}
#endif
