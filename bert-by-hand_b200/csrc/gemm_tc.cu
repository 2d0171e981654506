// Persistent tcgen05 GEMM for the encoder's four dense layers:
//   C[rows, N] = A[rows, K] . W[N, K]^T + bias   (+ erf-GELU | + residual, LayerNorm)
// Replaces the reference's wmma GEMM (src/kernels/matmul.cu:94-186) and, for the two
// N=384 projections, also its residual LayerNorm (src/kernels/layernorm.cu:17-59,
// called at src/model/encoder.cu:49-50 and :63-64).
//
// Design (sm_100a):
//  * one CTA per SM, persistent over 128 x BN output tiles (row count may be read from
//    device memory so a captured graph serves every batch shape);
//  * warp 0 = TMA producer (128B-swizzled K-major tiles into a STAGES-deep ring);
//  * warp 1 = MMA issuer: one thread issues tcgen05.mma kind::f16 (fp16 in, fp32 TMEM
//    accumulator), frees ring slots and publishes finished accumulators with
//    tcgen05.commit;
//  * warps 2.. = epilogue, 2 or 3 per TMEM lane quadrant (each a part of the columns):
//    tcgen05.ld 64 columns at a time, bias / GELU / residual + two-pass LayerNorm in
//    fp32 (row statistics combined through shared memory), fp16 stores. Two TMEM accumulators (when 2*BN <= 512)
//    let the MMA of tile i+1 overlap the epilogue of tile i.
#include <atomic>

#include "common.cuh"
#include "epilogue.cuh"
#include "internal.h"
#include "../../include/bbh.h"

#include <cstdio>
#include <cstring>
#include <mutex>

namespace bbh {

// Optional wait-time accounting for tuning (compiled only with -DBBH_GEMM_TRACE):
// [0] producer waiting for free ring slots, [1] MMA waiting for a free accumulator,
// [2] MMA waiting for operands, [3] epilogue waiting for a finished accumulator (one warp),
// [4] MMA-thread cycles from the first tile to the last commit, [5] tiles, [6] the same
// span in globaltimer ns; clock64 units otherwise.
#ifdef BBH_GEMM_TRACE
__device__ unsigned long long g_gemm_trace[8];
#define GEMM_TIMED(slot, expr)                   \
  ([&] {                                         \
    const long long t_ = clock64();              \
    const bool r_ = (expr);                      \
    trace_acc[slot] += clock64() - t_;           \
    return r_;                                   \
  }())
#else
#define GEMM_TIMED(slot, expr) (expr)
#endif

template <int BN, int EPI>
struct GemmCfg {
  static constexpr int BM = 128;
  static constexpr int BK = 64;  // 64 fp16 = one 128-byte swizzle row
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (160 * 1024) / STAGE_BYTES > 8 ? 8 : (160 * 1024) / STAGE_BYTES;
  static constexpr int NACC = (2 * BN <= 512) ? 2 : 1;
  static constexpr int TMEM_COLS = 512;  // power of two >= NACC*BN for every BN used here
  static constexpr int MMA_N = BN <= 256 ? BN : BN / 2;
  static constexpr int N_MMA = BN / MMA_N;
  static constexpr int TMA_B_ROWS = BN <= 256 ? BN : BN / 2;
  static constexpr int BIAS_COLS = EPI == kEpiResLN ? kHidden : kMaxBiasCols;
  static constexpr int AUX_BYTES = 256 /*barriers*/ + 4 * BIAS_COLS /*bias*/ +
                                   (EPI == kEpiResLN ? 8 * kHidden /*gamma, beta*/ +
                                                           2 * 2 * 3 * 128 * 4 /*row statistics, 2 slots*/ +
                                                           2048 /*peer statistics*/
                                                     : 0);
  // epilogue warps: 4 TMEM lane quadrants x PARTS column parts
  static constexpr int PARTS = BN == 192 ? 3 : 2;
  static constexpr int EPI_WARPS = 4 * PARTS;
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int STAGING_BYTES = EPI_WARPS * 4096;  // per warp: 32 rows x 128 B
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 /*align slack*/ + STAGING_BYTES + AUX_BYTES;
  static_assert(BN % 16 == 0 && MMA_N <= 256, "bad BN");
  static_assert(SMEM <= 227 * 1024, "shared memory over the per-CTA limit");
  static_assert(NACC * BN <= TMEM_COLS, "TMEM overflow");
  // The LayerNorm epilogue runs on a 2-CTA cluster: each CTA owns half of the 384-wide row
  // and the two exchange per-row statistics through distributed shared memory.
  static constexpr int CLUSTER = EPI == kEpiResLN ? 2 : 1;
  static_assert(EPI != kEpiResLN || BN * 2 == kHidden, "LayerNorm tiles are 128 x 192 per CTA");
};


template <int BN, int EPI>
__global__ void __launch_bounds__(GemmCfg<BN, EPI>::THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmR, GemmParams p) {
  using Cfg = GemmCfg<BN, EPI>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int NACC = Cfg::NACC;
  constexpr int HB = BN / Cfg::PARTS;  // columns per epilogue warp
  static_assert(HB % 32 == 0, "epilogue chunking");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES + Cfg::STAGING_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* accf_bar = empty_bar + STAGES;
  uint64_t* acce_bar = accf_bar + NACC;
  uint64_t* xfull_bar = acce_bar + NACC;  // [2] peer statistics arrived (cluster LayerNorm)
  uint64_t* res_bar = xfull_bar + 2;      // [EPI_WARPS] residual slice landed in staging (LayerNorm)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(res_bar + Cfg::EPI_WARPS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  uint8_t* s_stage = smem + STAGES * Cfg::STAGE_BYTES;  // epilogue staging, 1024-aligned
  float* s_bias = reinterpret_cast<float*>(s_stage + Cfg::STAGING_BYTES + 256);  // [BIAS_COLS]
  float* s_gamma = s_bias + Cfg::BIAS_COLS;                                          // [384]
  float* s_beta = s_gamma + kHidden;                                                 // [384]
  float* red = s_beta + kHidden;  // [2 slots][2 stats][3 parts][128 rows] (LayerNorm)
  float2* xstat = reinterpret_cast<float2*>(red + 2 * 2 * 3 * 128);  // [2 slots][128 rows] peer (mean, M2)

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
#ifdef BBH_GEMM_TRACE
  long long trace_acc[7] = {};
  const long long trace_t0 = clock64();
  const unsigned long long trace_g0 = globaltimer();
#endif

  pdl_launch_dependents();
  int rows = 0, m_tiles = 0;  // read after the wait for the previous kernel (below)
  const int n_tiles = (p.N + BN - 1) / BN;
  const int k_blocks = (p.K + Cfg::BK - 1) / Cfg::BK;
  // Tile schedule. Plain: tiles (m, n) in n-fastest order over all CTAs. Cluster: each
  // 2-CTA cluster walks m-tiles and CTA rank r owns columns [r*BN, (r+1)*BN).
  const int crank = Cfg::CLUSTER > 1 ? static_cast<int>(cluster_ctarank()) : 0;
  const int first_tile = Cfg::CLUSTER > 1 ? static_cast<int>(blockIdx.x) / 2 : static_cast<int>(blockIdx.x);
  const int tile_step = Cfg::CLUSTER > 1 ? static_cast<int>(gridDim.x) / 2 : static_cast<int>(gridDim.x);
  int num_tiles = 0;  // set once the row count is known
  auto tile_m0 = [&](int t) { return (Cfg::CLUSTER > 1 ? t : t / n_tiles) * Cfg::BM; };
  auto tile_n0 = [&](int t) { return Cfg::CLUSTER > 1 ? crank * BN : (t % n_tiles) * BN; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < NACC; ++a) {
      mbar_init(&accf_bar[a], 1);
      mbar_init(&acce_bar[a], Cfg::EPI_WARPS);  // one arrival per epilogue warp
    }
    // peer statistics: one local arrival (with the expected byte count) + 128 rows x 8 B
    // stored by the peer with st.async
    mbar_init(&xfull_bar[0], 1);
    mbar_init(&xfull_bar[1], 1);
    for (int w = 0; w < Cfg::EPI_WARPS; ++w) mbar_init(&res_bar[w], 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
    if constexpr (EPI == kEpiResLN) tma_prefetch_desc(&tmR);
  }
  if (warp == 1) tmem_alloc(tmem_holder, Cfg::TMEM_COLS);
  const bool bias_in_smem = p.bias && p.N <= Cfg::BIAS_COLS;
  if (bias_in_smem)
    for (int i = threadIdx.x; i < p.N; i += blockDim.x) s_bias[i] = __half2float(p.bias[i]);
  if constexpr (EPI == kEpiResLN) {
    for (int i = threadIdx.x; i < kHidden; i += blockDim.x) {
      s_gamma[i] = __half2float(p.gamma[i]);
      s_beta[i] = __half2float(p.beta[i]);
    }
  }
  // everything above touches only this kernel's own state and the weights; the
  // activations and the row count come from the previous kernel
  pdl_wait();
  rows = p.rows_dev ? *p.rows_dev : p.rows;
  m_tiles = (rows + Cfg::BM - 1) / Cfg::BM;
  num_tiles = Cfg::CLUSTER > 1 ? m_tiles : m_tiles * n_tiles;
  tc_fence_before();
  __syncthreads();
  if constexpr (Cfg::CLUSTER > 1) cluster_sync_all();  // peers' barriers are initialised
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = first_tile; tile < num_tiles && !*abort_flag; tile += tile_step) {
        const int m0 = tile_m0(tile);
        const int n0 = tile_n0(tile);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!GEMM_TIMED(0, mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag, p.err))) break;
          mbar_arrive_expect_tx(&full_bar[stage], Cfg::STAGE_BYTES);
          tma_load_2d(sA + stage * Cfg::A_BYTES, &tmA, &full_bar[stage], kb * Cfg::BK, m0);
#pragma unroll
          for (int h = 0; h < BN / Cfg::TMA_B_ROWS; ++h)
            tma_load_2d(sB + stage * Cfg::B_BYTES + h * Cfg::TMA_B_ROWS * 128, &tmB, &full_bar[stage],
                        kb * Cfg::BK, n0 + h * Cfg::TMA_B_ROWS);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(128, Cfg::MMA_N);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int tile = first_tile; tile < num_tiles && !*abort_flag; tile += tile_step) {
        if (!GEMM_TIMED(1, mbar_wait(&acce_bar[acc], acc_phase ^ 1, abort_flag, p.err))) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!GEMM_TIMED(2, mbar_wait(&full_bar[stage], phase, abort_flag, p.err))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * Cfg::A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * Cfg::B_BYTES);
#pragma unroll
          for (int k = 0; k < Cfg::BK / 16; ++k) {
            const uint64_t adesc = sw128_kmajor_desc(a_addr + k * 32);
#pragma unroll
            for (int h = 0; h < Cfg::N_MMA; ++h) {
              const uint64_t bdesc = sw128_kmajor_desc(b_addr + h * Cfg::MMA_N * 128 + k * 32);
              tc_mma_f16(d_tmem + h * Cfg::MMA_N, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
            }
          }
          tc_commit(&empty_bar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit(&accf_bar[acc]);
#ifdef BBH_GEMM_TRACE
        trace_acc[4] = clock64() - trace_t0;
        trace_acc[5] += 1;
        trace_acc[6] = static_cast<long long>(globaltimer() - trace_g0);
#endif
        if (++acc == NACC) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..9)
    const int quad = warp & 3;        // TMEM lane quadrant this warp may access
    const int half = (warp - 2) >> 2;  // which column part of the tile (0 .. PARTS-1)
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    ChunkStore cst{s_stage + (warp - 2) * 4096, &tmC, lane};
    int acc = 0;
    uint32_t acc_phase = 0;
    int iter = 0;  // tiles processed by this CTA (peer-statistics slot and phase)
    const int we = warp - 2;  // epilogue warp index
    // LayerNorm: the residual slice of the first tile is queued before the loop
    const LnSlice ln{cst.buf, &tmC, &tmR, &res_bar[we], red, xstat, xfull_bar,
                     static_cast<uint32_t>(crank ^ 1), s_bias, s_gamma, s_beta, p.eps, lane, quad, half, we};
    if constexpr (EPI == kEpiResLN) {
      if (first_tile < num_tiles) ln.prefetch(tile_n0(first_tile) + half * HB, tile_m0(first_tile) + quad * 32);
    }
    for (int tile = first_tile; tile < num_tiles; tile += tile_step, ++iter) {
      const int m0 = tile_m0(tile);
      const int c0 = tile_n0(tile) + half * HB;  // first output column of this warp
      if (!GEMM_TIMED(3, mbar_wait(&accf_bar[acc], acc_phase, abort_flag, p.err))) break;
      tc_fence_after();
      const uint32_t tacc = tmem_base + lane_off + acc * BN + half * HB;
      const int row0 = m0 + quad * 32;  // first row of this warp's 32-row slab

      if constexpr (EPI == kEpiResLN) {
        static_assert(HB == 64, "LayerNorm epilogue: 64 columns per warp");
        // the accumulator slice, then hand the accumulator straight back to the MMA warp
        float v[64];
        tmem_ld64(tacc, tacc + 32, v);
        warp_arrive(&acce_bar[acc]);
        const int nt = tile + tile_step;
        if (!ln.finish(v, iter, c0, row0, nt < num_tiles, tile_n0(nt) + half * HB, tile_m0(nt) + quad * 32, abort_flag,
                       p.err))
          break;
      } else {
        const float* sb = bias_in_smem ? s_bias : nullptr;
        static_assert(HB % 64 == 0, "64-column output chunks");
#pragma unroll 1
        for (int c = 0; c < HB; c += 64) {
          float v[64];
          tmem_ld64(tacc + c, tacc + c + 32, v);
          if (c + 64 >= HB) warp_arrive(&acce_bar[acc]);  // accumulator fully read
          uint32_t w[32];
          epi_pack32<EPI>(v, c0 + c, sb, p.bias, p.N, w);
          epi_pack32<EPI>(v + 32, c0 + c + 32, sb, p.bias, p.N, w + 16);
          cst.put64(w, c0 + c, row0);
        }
      }
      if (++acc == NACC) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    cst.drain();
  }

#ifdef BBH_GEMM_TRACE
  if (lane == 0 && warp <= 2)
    for (int i = 0; i < 7; ++i) atomicAdd(&g_gemm_trace[i], static_cast<unsigned long long>(trace_acc[i]));
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
  if constexpr (Cfg::CLUSTER > 1) cluster_sync_all();  // no peer still writes into this CTA
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ======================================================================== host side

typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled get_encode_fn() {
  static PFN_encodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled>(ptr);
  });
  return fn;
}

// Row-major [rows, cols] fp16 matrix with row stride ld elements; box = box_cols x box_rows
// with the given swizzle (operands: 64 x rows, 128-byte swizzle, matching
// sw128_kmajor_desc; outputs: 32 x 32, 64-byte swizzle, matching ChunkStore).
int encode_2d(CUtensorMap* map, const __half* base, int rows, int cols, int ld, int box_cols, int box_rows,
              CUtensorMapSwizzle swz) {
  PFN_encodeTiled enc = get_encode_fn();
  if (!enc) return BBH_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld * 2) % 16) return BBH_ERR_ARG;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? BBH_OK : BBH_ERR_CUDA;
}

template <int BN, int EPI>
static cudaError_t launch_inst(const GemmPlan& plan, cudaStream_t stream, bool pdl) {
  using Cfg = GemmCfg<BN, EPI>;
  static bool attr_set[64] = {};
  static int max_clusters[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  auto kern = gemm_tc_kernel<BN, EPI>;
  if (dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
    if (e != cudaSuccess) return e;
    if constexpr (Cfg::CLUSTER > 1) {
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 0);
      (void)e;
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
    }
    attr_set[dev] = true;
  }
  if constexpr (Cfg::CLUSTER > 1) {
    const int m_tiles_cap = (plan.rows_cap + Cfg::BM - 1) / Cfg::BM;
    int nclusters = dev < 64 ? max_clusters[dev] : 64;
    if (nclusters > m_tiles_cap) nclusters = m_tiles_cap;
    return launch_ex(kern, dim3(Cfg::CLUSTER * nclusters), dim3(Cfg::THREADS), Cfg::SMEM, stream, pdl, Cfg::CLUSTER,
                     plan.tmA, plan.tmB, plan.tmC, plan.tmR, plan.p);
  } else {
    return launch_ex(kern, dim3(plan.grid), dim3(Cfg::THREADS), Cfg::SMEM, stream, pdl, 1, plan.tmA, plan.tmB,
                     plan.tmC, plan.tmR, plan.p);
  }
}

int make_gemm_plan(GemmPlan* plan, const __half* A, int lda, int rows_cap, const __half* W, int N, int K,
                   __half* C, int ldc, int epi, int num_sms, int pair_mode) {
  if (!plan || !A || !W || !C || rows_cap <= 0 || N <= 0 || K <= 0 || N % 8 || K % 8 || lda < K || ldc < N)
    return BBH_ERR_ARG;
  int bn;
  if (epi == kEpiResLN) {
    if (N != kHidden) return BBH_ERR_ARG;
    bn = 192;  // per CTA of a 2-CTA cluster
  } else if (N % 192 == 0) {
    bn = 192;  // three epilogue warps per TMEM quadrant
  } else if (N % 256 == 0) {
    bn = 256;
  } else {
    bn = 128;
  }
  const int box_b = bn;
  memset(&plan->tmR, 0, sizeof(plan->tmR));
  int rc = encode_2d(&plan->tmA, A, rows_cap, K, lda, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = encode_2d(&plan->tmB, W, N, K, K, 64, box_b, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = encode_2d(&plan->tmC, C, rows_cap, N, ldc, 64, 32, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  plan->bn = bn;
  plan->bn2 = 0;
  memset(&plan->tmB2, 0, sizeof(plan->tmB2));
  // The residual-LayerNorm pair kernel gives each SM pair a whole 256-row tile; when a
  // launch has fewer such tiles than SM pairs (small batches), the one-SM kernel's 128-row
  // tiles on 2-CTA clusters keep more SMs busy (the two give bit-identical results).
  const bool ln_small = epi == kEpiResLN && (rows_cap + 255) / 256 < num_sms / 2;
  if (pair_mode && !ln_small) {
    const int order[2] = {pair_mode == 2 ? 256 : 192, pair_mode == 2 ? 192 : 256};
    for (int b2 : order)
      if (gemm_pair_supported(N, epi, b2)) {
        rc = encode_2d(&plan->tmB2, W, N, K, K, 64, b2 / 2, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
        plan->bn2 = b2;
        break;
      }
  }
  plan->epi = epi;
  plan->rows_cap = rows_cap;
  const int tiles_cap = ((rows_cap + 127) / 128) * ((N + bn - 1) / bn);
  plan->grid = tiles_cap < num_sms ? tiles_cap : num_sms;
  GemmParams& p = plan->p;
  p = GemmParams{};
  p.N = N;
  p.K = K;
  p.C = C;
  p.ldc = ldc;
  p.eps = 1e-12f;
  return BBH_OK;
}

int set_gemm_residual(GemmPlan* plan, const __half* R, int ldr) {
  if (!plan || !R || ldr < plan->p.N) return BBH_ERR_ARG;
  plan->p.residual = R;
  plan->p.ldr = ldr;
  // 32 x 64 boxes in the output chunks' 128-byte-swizzle layout
  return encode_2d(&plan->tmR, R, plan->rows_cap, plan->p.N, ldr, 64, 32, CU_TENSOR_MAP_SWIZZLE_128B);
}

static std::atomic<int> g_default_pair_mode{2};
int default_gemm_pair_mode() { return g_default_pair_mode.load(std::memory_order_relaxed); }
void set_default_gemm_pair_mode(int mode) { g_default_pair_mode.store(mode, std::memory_order_relaxed); }

cudaError_t launch_gemm(const GemmPlan& plan, cudaStream_t stream, bool pdl) {
  if (plan.epi == kEpiResLN && !plan.p.residual) return cudaErrorInvalidValue;
  if (plan.bn2) return launch_gemm_pair(plan, stream, pdl);
  switch (plan.epi * 1000 + plan.bn) {
    case kEpiBias * 1000 + 128: return launch_inst<128, kEpiBias>(plan, stream, pdl);
    case kEpiGelu * 1000 + 128: return launch_inst<128, kEpiGelu>(plan, stream, pdl);
    case kEpiBias * 1000 + 192: return launch_inst<192, kEpiBias>(plan, stream, pdl);
    case kEpiGelu * 1000 + 192: return launch_inst<192, kEpiGelu>(plan, stream, pdl);
    case kEpiBias * 1000 + 256: return launch_inst<256, kEpiBias>(plan, stream, pdl);
    case kEpiGelu * 1000 + 256: return launch_inst<256, kEpiGelu>(plan, stream, pdl);
    case kEpiResLN * 1000 + 192: return launch_inst<192, kEpiResLN>(plan, stream, pdl);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace bbh
