// CTA-pair (cta_group::2) tcgen05 GEMM for the encoder's bias / GELU projections:
//   C[rows, N] = A[rows, K] . W[N, K]^T + bias   (+ erf-GELU)
// i.e. the fused QKV projection (N = 1152) and the first FFN layer (N = 1536, GELU): the
// reference's wmma GEMM (src/kernels/matmul.cu:94-186) followed by its bias / GELU
// kernels. The two N = 384 projections with the residual LayerNorm run on gemm_ln.cu.
//
// Why pairs: with one SM per 128 x BN tile every SM streams its own copy of the B tile
// (BN x 64 per k-block) from L2 next to its A tile, and at full tensor rate that L2 ->
// shared-memory traffic is the limit. Two SMs of a cluster working one 256 x BN tile with
// one M=256 MMA each hold 128 A rows and only BN/2 B rows, so the operand bytes per FLOP
// drop by 1.4x (BN=192) to 1.6x (BN=256) at the same accumulator size per SM.
//
// Roles (both CTAs of a pair run every role except the MMA issue):
//  * warp 0 lane 0: TMA producer for this CTA's halves (A rows, B rows) of each k-block;
//    the bytes of both CTAs complete on the EVEN CTA's full barrier;
//  * warp 1: TMEM allocation for the pair; in the even CTA lane 0 also issues the M=256
//    MMAs and commits to both CTAs' ring-slot and accumulator barriers;
//  * warps 2..: epilogue over this CTA's 128 accumulator rows (bias, GELU, fp16, TMA
//    stores); each warp's release of an accumulator arrives on the even CTA's barrier.
// Every wait is bounded (mbar_wait*), exactly as in the one-SM kernel.
#include "common.cuh"
#include "epilogue.cuh"
#include "internal.h"
#include "../../include/bbh.h"

namespace bbh {

template <int BN, int PARTS, int EPI>
struct PairCfg {
  static_assert(EPI == kEpiBias || EPI == kEpiGelu, "bias / GELU epilogues");
  static constexpr int CLUSTER = 2;
  static constexpr int BM = 128;           // accumulator rows per CTA (256 per pair)
  static constexpr int BK = 64;            // one 128-byte swizzle row of fp16
  static constexpr int B_ROWS = BN / 2;    // B rows held by each CTA
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = B_ROWS * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int EPI_WARPS = 4 * PARTS;
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int STAGING_BYTES = EPI_WARPS * 4096;  // per epilogue warp: 32 rows x 128 B
  static constexpr int BIAS_COLS = kMaxBiasCols;
  static constexpr int AUX_BYTES = 512 /*barriers*/ + 4 * BIAS_COLS;
  static constexpr int RING_BYTES = 227 * 1024 - 1024 - STAGING_BYTES - AUX_BYTES;
  static constexpr int STAGES = RING_BYTES / STAGE_BYTES > 8 ? 8 : RING_BYTES / STAGE_BYTES;
  static constexpr int NACC = 2;
  static constexpr int TMEM_COLS = 512;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + STAGING_BYTES + AUX_BYTES;
  static_assert(BN % 32 == 0 && BN <= 256, "pair MMA: N <= 256, B halves of whole 16-row groups");
  static_assert((BN / PARTS) % 64 == 0, "64-column output chunks");
  static_assert(NACC * BN <= TMEM_COLS, "TMEM overflow");
  static_assert(STAGES >= 3, "operand ring too shallow");
  static_assert(SMEM <= 227 * 1024, "shared memory over the per-CTA limit");
};

template <int BN, int EPI, int PARTS>
__global__ void __launch_bounds__(PairCfg<BN, PARTS, EPI>::THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, GemmParams p) {
  using Cfg = PairCfg<BN, PARTS, EPI>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int NACC = Cfg::NACC;
  constexpr int HB = BN / PARTS;  // columns per epilogue warp

  extern __shared__ uint8_t smem_raw[];
  // the same 1024-aligned offsets in both CTAs: the pair MMA reads both at one address
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  uint8_t* s_stage = smem + STAGES * Cfg::STAGE_BYTES;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(s_stage + Cfg::STAGING_BYTES);  // used in the even CTA
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* accf_bar = empty_bar + STAGES;
  uint64_t* acce_bar = accf_bar + NACC;  // used in the even CTA
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acce_bar + NACC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* s_bias = reinterpret_cast<float*>(s_stage + Cfg::STAGING_BYTES + 512);  // [BIAS_COLS]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();
  const uint32_t lead_rank = crank & ~1u;  // even CTA of this CTA's pair
  const bool leader = crank == lead_rank;
  const int half = static_cast<int>(crank & 1);  // which 128 rows of the pair tile

  pdl_launch_dependents();
  const int n_tiles = (p.N + BN - 1) / BN;
  const int k_blocks = (p.K + Cfg::BK - 1) / Cfg::BK;
  const int first_tile = static_cast<int>(blockIdx.x) / Cfg::CLUSTER;  // one tile per cluster at a time
  const int tile_step = static_cast<int>(gridDim.x) / Cfg::CLUSTER;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);   // the even CTA's producer arrival (+ both CTAs' bytes)
      mbar_init(&empty_bar[s], 1);  // one commit from the MMA thread
    }
    for (int a = 0; a < NACC; ++a) {
      mbar_init(&accf_bar[a], 1);
      mbar_init(&acce_bar[a], 2 * Cfg::EPI_WARPS);  // every epilogue warp of both CTAs
    }
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
  }
  if (warp == 1) tmem_alloc_pair(tmem_holder, Cfg::TMEM_COLS);
  const bool bias_in_smem = p.bias && p.N <= Cfg::BIAS_COLS;
  if (bias_in_smem)
    for (int i = threadIdx.x; i < p.N; i += blockDim.x) s_bias[i] = __half2float(p.bias[i]);
  pdl_wait();
  const int rows = p.rows_dev ? *p.rows_dev : p.rows;
  const int m_pairs = (rows + 2 * Cfg::BM - 1) / (2 * Cfg::BM);
  const int num_tiles = m_pairs * n_tiles;
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // every CTA's barriers initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  // tile t: rows [256 * m, +256) with this CTA's 128 at +128 * half; columns [n0, +BN),
  // (m, n0) = (t / n_tiles, BN * (t % n_tiles))
  auto tile_m0 = [&](int t) { return (t / n_tiles) * (2 * Cfg::BM) + half * Cfg::BM; };
  auto tile_n0 = [&](int t) { return (t % n_tiles) * BN; };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      const uint32_t full0 = mapa_shared(smem_u32(full_bar), lead_rank);
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = first_tile; tile < num_tiles && !*abort_flag; tile += tile_step) {
        const int m0 = tile_m0(tile);
        const int nb = tile_n0(tile) + half * Cfg::B_ROWS;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag, p.err)) break;
          // the even CTA announces both CTAs' bytes; the odd CTA's copies may land first
          // (the transaction count may go transiently negative within a phase)
          if (leader) mbar_arrive_expect_tx(&full_bar[stage], 2 * Cfg::STAGE_BYTES);
          const uint32_t fb = full0 + stage * 8;
          tma_load_2d_pair(sA + stage * Cfg::A_BYTES, &tmA, fb, kb * Cfg::BK, m0);
          tma_load_2d_pair(sB + stage * Cfg::B_BYTES, &tmB, fb, kb * Cfg::BK, nb);
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
      constexpr uint32_t idesc = idesc_f16_f32(2 * Cfg::BM, BN);
      const uint32_t empty_peer = mapa_shared(smem_u32(empty_bar), crank + 1);
      const uint32_t accf_peer = mapa_shared(smem_u32(accf_bar), crank + 1);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int tile = first_tile; tile < num_tiles && !*abort_flag; tile += tile_step) {
        if (!mbar_wait(&acce_bar[acc], acc_phase ^ 1, abort_flag, p.err)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * Cfg::A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * Cfg::B_BYTES);
#pragma unroll
          for (int k = 0; k < Cfg::BK / 16; ++k)
            tc_mma_f16_pair(d_tmem, sw128_kmajor_desc(a_addr + k * 32), sw128_kmajor_desc(b_addr + k * 32), idesc,
                            (kb | k) != 0 ? 1u : 0u);
          // the slot is free in both CTAs once these MMAs have read it
          tc_commit_pair(smem_u32(&empty_bar[stage]));
          tc_commit_pair(empty_peer + stage * 8);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit_pair(smem_u32(&accf_bar[acc]));
        tc_commit_pair(accf_peer + acc * 8);
        if (++acc == NACC) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int quad = warp & 3;             // TMEM lane quadrant this warp may access
    const int part = (warp - 2) >> 2;      // column part of the tile (0 .. PARTS-1)
    const int we = warp - 2;               // epilogue warp index
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    ChunkStore cst{s_stage + we * 4096, &tmC, lane};
    const uint32_t acce0 = mapa_shared(smem_u32(acce_bar), lead_rank);
    const float* sb = bias_in_smem ? s_bias : nullptr;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = first_tile; tile < num_tiles; tile += tile_step) {
      if (!mbar_wait(&accf_bar[acc], acc_phase, abort_flag, p.err)) break;
      tc_fence_after();
      const uint32_t tacc = tmem_base + lane_off + acc * BN + part * HB;
      const int row0 = tile_m0(tile) + quad * 32;
      const int c0 = tile_n0(tile) + part * HB;
#pragma unroll 1
      for (int c = 0; c < HB; c += 64) {
        float v[64];
        tmem_ld64(tacc + c, tacc + c + 32, v);
        if (c + 64 >= HB) {
          // accumulator fully read by this warp: release it to the even CTA's MMA thread
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(acce0 + acc * 8);
        }
        uint32_t w[32];
        epi_pack32<EPI>(v, c0 + c, sb, p.bias, p.N, w);
        epi_pack32<EPI>(v + 32, c0 + c + 32, sb, p.bias, p.N, w + 16);
        cst.put64(w, c0 + c, row0);
      }
      if (++acc == NACC) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    cst.drain();
  }

  tc_fence_before();
  __syncthreads();
  if (*abort_flag && warp == 0 && lane == 0) {
    // Let in-flight TMA copies land before the CTA's shared memory is released.
    const unsigned long long t0 = globaltimer();
    while (globaltimer() - t0 < 1000000ull) {
    }
  }
  __syncthreads();
  cluster_sync_all();  // no other CTA of the cluster still reads or signals this CTA's memory
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
}

// ======================================================================== host side

template <int BN, int EPI, int PARTS>
static cudaError_t launch_pair_inst(const GemmPlan& plan, cudaStream_t stream, bool pdl) {
  using Cfg = PairCfg<BN, PARTS, EPI>;
  static bool attr_set[64] = {};
  static int max_clusters[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  auto kern = gemm_pair_kernel<BN, EPI, PARTS>;
  if (dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = Cfg::CLUSTER;
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
  const int m_pairs = (plan.rows_cap + 255) / 256;
  const int tiles_cap = m_pairs * ((plan.p.N + BN - 1) / BN);
  int nclusters = dev < 64 ? max_clusters[dev] : 64;
  if (nclusters > tiles_cap) nclusters = tiles_cap;
  return launch_ex(kern, dim3(Cfg::CLUSTER * nclusters), dim3(Cfg::THREADS), Cfg::SMEM, stream, pdl, Cfg::CLUSTER,
                   plan.tmA, plan.tmB2, plan.tmC, plan.p);
}

bool gemm_pair_supported(int N, int epi, int bn) {
  if (epi == kEpiResLN) return N == kHidden && bn == 192;
  if (epi != kEpiBias && epi != kEpiGelu) return false;
  return (bn == 192 || bn == 256) && N % bn == 0;
}

cudaError_t launch_gemm_pair(const GemmPlan& plan, cudaStream_t stream, bool pdl) {
  switch (plan.epi * 1000 + plan.bn2) {
    case kEpiBias * 1000 + 192: return launch_pair_inst<192, kEpiBias, 3>(plan, stream, pdl);
    case kEpiGelu * 1000 + 192: return launch_pair_inst<192, kEpiGelu, 3>(plan, stream, pdl);
    case kEpiBias * 1000 + 256: return launch_pair_inst<256, kEpiBias, 4>(plan, stream, pdl);
    case kEpiGelu * 1000 + 256: return launch_pair_inst<256, kEpiGelu, 4>(plan, stream, pdl);
    case kEpiResLN * 1000 + 192: return launch_gemm_ln_pair(plan, stream, pdl);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace bbh
