// Fused feed-forward block: out = LayerNorm(GELU(Y W1^T + b1) W2^T + b2 + Y) * gamma + beta
// in one persistent kernel. Replaces the reference's ffn_block (src/model/encoder.cu:52-64:
// FFN1 GEMM with GELU into a [rows, 1536] buffer, FFN2 GEMM, residual LayerNorm -- three
// launches and a 3 KB-per-token round trip of the intermediate through HBM).
//
// Per 128-row tile (one CTA per SM, persistent over tiles):
//   * the 1536 intermediate columns are produced in 12 chunks of 128: MMA1 computes the
//     chunk (K = 384) into a 128-column TMEM accumulator; the epilogue warps add b1, apply
//     GELU on fp16 pairs and write the chunk to shared memory as a 128-byte-swizzled
//     K-major operand (two buffers, alternating by chunk); MMA2 accumulates
//     chunk . W2[:, chunk]^T into the 384-column FFN2 accumulator in TMEM. The
//     intermediate never leaves the SM.
//   * after the last chunk the epilogue adds b2 and the residual, writes that back into
//     TMEM while taking shifted row sums, combines the four column parts of every row
//     through shared memory, then normalises and stores.
// Measured on B200 (cfg3 batch, T = 68,451): 250 us against ~211 us for the two GEMM
// launches it replaces, so the workspace forward keeps the two GEMMs by default
// (bbh_ws_set_ffn_fusion). The tensor core alone needs ~138 us here: MMA1's 128-column
// chunks and MMA2's three 128-column products read their shared-memory operands at a
// lower FLOP/byte than the GEMMs' 192-column tiles, and each MMA1 K block streams 32 KB
// (the Y and W1 boxes), more than an 8-entry ring hides. A 2-SM (cta_group::2) version that
// halves the per-SM weight traffic is the way to make the fusion pay.
// Roles: warp 0 = TMA producer (one ring of 16 KB entries shared by both MMAs, filled in
// the order the MMA warp consumes it), warp 1 = MMA issuer (one thread), warps 2..17 =
// epilogue (4 per TMEM lane quadrant, 32 columns each of a chunk, 96 of the LayerNorm).
#include "common.cuh"
#include "epilogue.cuh"
#include "internal.h"
#include "../../include/bbh.h"

#include <cstring>

namespace bbh {

namespace {

constexpr int kBM = 128;               // rows per tile
constexpr int kCh = 128;               // intermediate columns per chunk
constexpr int kNch = kFfn / kCh;       // 12 chunks
constexpr int kKb1 = kHidden / 64;     // MMA1 K blocks (64 wide)
constexpr int kKb2 = kCh / 64;         // MMA2 K blocks per chunk
constexpr int kSlot = 16 * 1024;       // ring entry: one 128-row x 64-column TMA box
constexpr int kSlots = 8;              // MMA1 K block = 2 entries (Y, W1), MMA2 K block = 3 (W2 rows)
constexpr int kHbuf = kBM * kCh * 2;   // 32 KB per intermediate chunk buffer
constexpr int kEpiWarps = 16;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kAuxBytes = 256 /*barriers*/ + 4 * kFfn /*b1*/ + 3 * 4 * kHidden /*b2, gamma, beta*/ +
                          2 * 4 * kBM * 4 /*row statistics*/;
constexpr int kSmem = 1024 + kSlots * kSlot + 2 * kHbuf + kAuxBytes;
static_assert(kSmem <= 227 * 1024, "shared memory over the per-CTA limit");
constexpr uint32_t kAcc2Col = 0;    // FFN2 accumulator: TMEM columns [0, 384)
constexpr uint32_t kHaccCol = 384;  // chunk accumulator: [384, 512)

}  // namespace

// Optional wait-time accounting for tuning (compiled only with -DBBH_MLP_TRACE), clock64
// units summed over CTAs: [0] producer waiting for ring entries, [1] MMA waiting for the
// chunk accumulator, [2] MMA waiting for operands, [3] MMA waiting for an intermediate
// chunk, [4] MMA waiting for the FFN2 accumulator, [5] epilogue waiting for a chunk
// accumulator, [6] epilogue waiting for a free chunk buffer, [7] epilogue waiting for the
// FFN2 accumulator, [8] LayerNorm epilogue, [9] MMA-thread span, [10] tiles.
#ifdef BBH_MLP_TRACE
__device__ unsigned long long g_mlp_trace[12];
#define MLP_TIMED(slot, expr)          \
  ([&] {                               \
    const long long t_ = clock64();    \
    const bool r_ = (expr);            \
    trace_acc[slot] += clock64() - t_; \
    return r_;                         \
  }())
#else
#define MLP_TIMED(slot, expr) (expr)
#endif

__global__ void __launch_bounds__(kThreads, 1)
    mlp_fused_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW1,
                     const __grid_constant__ CUtensorMap tmW2, MlpParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint8_t* hbuf = ring + kSlots * kSlot;  // [2][2 K blocks][128 rows][128 B]
  uint64_t* full = reinterpret_cast<uint64_t*>(hbuf + 2 * kHbuf);
  uint64_t* empty = full + kSlots;
  uint64_t* hacc_full = empty + kSlots;
  uint64_t* hacc_free = hacc_full + 1;
  uint64_t* h_ready = hacc_free + 1;   // [2]
  uint64_t* hbuf_free = h_ready + 2;   // [2]
  uint64_t* acc2_full = hbuf_free + 2;
  uint64_t* acc2_free = acc2_full + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acc2_free + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* s_b1 = reinterpret_cast<float*>(hbuf + 2 * kHbuf + 256);
  float* s_b2 = s_b1 + kFfn;
  float* s_gamma = s_b2 + kHidden;
  float* s_beta = s_gamma + kHidden;
  float* red = s_beta + kHidden;  // [2 stats][4 parts][128 rows]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
#ifdef BBH_MLP_TRACE
  long long trace_acc[12] = {};
  const long long trace_t0 = clock64();
#endif
  pdl_launch_dependents();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(hacc_full, 1);
    mbar_init(hacc_free, kEpiWarps);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&h_ready[b], kEpiWarps);
      mbar_init(&hbuf_free[b], 1);
    }
    mbar_init(acc2_full, 1);
    mbar_init(acc2_free, kEpiWarps);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW1);
    tma_prefetch_desc(&tmW2);
  }
  if (warp == 1) tmem_alloc(tmem_holder, 512);
  for (int i = threadIdx.x; i < kFfn; i += blockDim.x) s_b1[i] = __half2float(p.b1[i]);
  for (int i = threadIdx.x; i < kHidden; i += blockDim.x) {
    s_b2[i] = __half2float(p.b2[i]);
    s_gamma[i] = __half2float(p.gamma[i]);
    s_beta[i] = __half2float(p.beta[i]);
  }
  pdl_wait();  // the activations and the row count come from the previous kernel
  const int rows = p.rows_dev ? *p.rows_dev : p.rows;
  const int m_tiles = (rows + kBM - 1) / kBM;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int slot = 0;
      uint32_t ph = 0;
      auto next = [&]() {
        if (++slot == kSlots) {
          slot = 0;
          ph ^= 1;
        }
      };
      auto load = [&](const CUtensorMap* map, int x, int y) -> bool {
        if (!MLP_TIMED(0, mbar_wait(&empty[slot], ph ^ 1, abort_flag, p.err))) return false;
        mbar_arrive_expect_tx(&full[slot], kSlot);
        tma_load_2d(ring + slot * kSlot, map, &full[slot], x, y);
        next();
        return true;
      };
      auto load_mma1 = [&](int m0, int j) -> bool {
        for (int kb = 0; kb < kKb1; ++kb)
          if (!load(&tmX, kb * 64, m0) || !load(&tmW1, kb * 64, j * kCh)) return false;
        return true;
      };
      auto load_mma2 = [&](int j) -> bool {
        for (int kb = 0; kb < kKb2; ++kb)
          for (int r = 0; r < 3; ++r)
            if (!load(&tmW2, j * kCh + kb * 64, r * 128)) return false;
        return true;
      };
      bool ok = true;
      for (int tile = blockIdx.x; tile < m_tiles && ok; tile += gridDim.x) {
        const int m0 = tile * kBM;
        for (int j = 0; j < kNch && ok; ++j) {
          ok = load_mma1(m0, j);
          if (ok && j > 0) ok = load_mma2(j - 1);
        }
        if (ok) ok = load_mma2(kNch - 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc1 = idesc_f16_f32(128, kCh);
      constexpr uint32_t idesc2 = idesc_f16_f32(128, 128);
      const uint32_t hacc = tmem_base + kHaccCol;
      const uint32_t acc2 = tmem_base + kAcc2Col;
      int slot = 0;
      uint32_t ph = 0;
      uint32_t hacc_n = 0, h_n[2] = {0, 0}, tile_n = 0;
      auto next = [&]() {
        if (++slot == kSlots) {
          slot = 0;
          ph ^= 1;
        }
      };
      auto mma1 = [&](int j) -> bool {
        (void)j;
        if (!MLP_TIMED(1, mbar_wait(hacc_free, (hacc_n & 1) ^ 1, abort_flag, p.err))) return false;
        tc_fence_after();
        for (int kb = 0; kb < kKb1; ++kb) {
          const int sa = slot;
          if (!MLP_TIMED(2, mbar_wait(&full[sa], ph, abort_flag, p.err))) return false;
          next();
          const int sb = slot;
          if (!MLP_TIMED(2, mbar_wait(&full[sb], ph, abort_flag, p.err))) return false;
          next();
          tc_fence_after();
          const uint32_t a = smem_u32(ring + sa * kSlot), b = smem_u32(ring + sb * kSlot);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            tc_mma_f16(hacc, sw128_kmajor_desc(a + k * 32), sw128_kmajor_desc(b + k * 32), idesc1, (kb | k) != 0);
          tc_commit(&empty[sa]);
          tc_commit(&empty[sb]);
        }
        tc_commit(hacc_full);
        ++hacc_n;
        return true;
      };
      auto mma2 = [&](int j) -> bool {
        const int hb = j & 1;
        if (j == 0) {
          if (!MLP_TIMED(4, mbar_wait(acc2_free, (tile_n & 1) ^ 1, abort_flag, p.err))) return false;
        }
        if (!MLP_TIMED(3, mbar_wait(&h_ready[hb], h_n[hb] & 1, abort_flag, p.err))) return false;
        tc_fence_after();
        const uint32_t h = smem_u32(hbuf + hb * kHbuf);
        for (int kb = 0; kb < kKb2; ++kb) {
          int sw[3];
          for (int r = 0; r < 3; ++r) {
            sw[r] = slot;
            if (!MLP_TIMED(2, mbar_wait(&full[slot], ph, abort_flag, p.err))) return false;
            next();
          }
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t adesc = sw128_kmajor_desc(h + kb * 16384 + k * 32);
            const uint32_t acc = (j | kb | k) != 0;
#pragma unroll
            for (int r = 0; r < 3; ++r)
              tc_mma_f16(acc2 + r * 128, adesc, sw128_kmajor_desc(smem_u32(ring + sw[r] * kSlot) + k * 32), idesc2,
                         acc);
          }
          for (int r = 0; r < 3; ++r) tc_commit(&empty[sw[r]]);
        }
        tc_commit(&hbuf_free[hb]);
        ++h_n[hb];
        return true;
      };
      bool ok = true;
      for (int tile = blockIdx.x; tile < m_tiles && ok; tile += gridDim.x) {
        for (int j = 0; j < kNch && ok; ++j) {
          ok = mma1(j);
          if (ok && j > 0) ok = mma2(j - 1);
        }
        if (ok) ok = mma2(kNch - 1);
        if (ok) {
          tc_commit(acc2_full);
          ++tile_n;
#ifdef BBH_MLP_TRACE
          trace_acc[9] = clock64() - trace_t0;
          trace_acc[10] += 1;
#endif
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..17)
    const int quad = warp & 3;             // TMEM lane quadrant this warp may access
    const int part = (warp - 2) >> 2;      // column part 0..3
    const int rloc = quad * 32 + lane;     // row within the tile
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t hacc = tmem_base + lane_off + kHaccCol + part * 32;
    const uint32_t acc2 = tmem_base + lane_off + kAcc2Col + part * 96;
    uint32_t hacc_n = 0, h_n[2] = {0, 0}, tile_n = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < m_tiles && ok; tile += gridDim.x) {
      const int m0 = tile * kBM;
      for (int j = 0; j < kNch; ++j) {
        const int hb = j & 1;
        if (!MLP_TIMED(5, mbar_wait(hacc_full, hacc_n & 1, abort_flag, p.err))) {
          ok = false;
          break;
        }
        tc_fence_after();
        float v[32];
        tmem_ld32(hacc, v);
        warp_arrive(hacc_free);
        ++hacc_n;
        if (!MLP_TIMED(6, mbar_wait(&hbuf_free[hb], (h_n[hb] & 1) ^ 1, abort_flag, p.err))) {
          ok = false;
          break;
        }
        uint32_t w[16];
        epi_pack32<kEpiGelu>(v, j * kCh + part * 32, s_b1, nullptr, kFfn, w);
        // 32 columns = 4 pieces of 16 B in K block part/2, pieces (part&1)*4 .. +3
        uint8_t* rowp = hbuf + hb * kHbuf + (part >> 1) * 16384 + rloc * 128;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int c = (part & 1) * 4 + i;
          *reinterpret_cast<uint4*>(rowp + ((c ^ (rloc & 7)) << 4)) =
              make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
        }
        fence_async_shared();  // generic stores -> visible to the tensor core
        warp_arrive(&h_ready[hb]);
        ++h_n[hb];
      }
      if (!ok) break;
      // ---- residual LayerNorm over the 384 columns of the tile's rows. The residual and the
      // output move through a 2 KB per-warp staging area (in the idle intermediate
      // buffer) so that global accesses are whole 64-byte row pieces: lane l handles row
      // 8i + l/4, 16-byte piece l%4 of the warp's 32 x 32 block (four instructions).
      uint8_t* stg = hbuf + (warp - 2) * 2048;  // 32 rows x 64 B, piece c of row r at c ^ ((r >> 1) & 3)
      const int crow = lane >> 2, cpiece = lane & 3;
      auto stg_at = [&](int r, int c) { return stg + r * 64 + ((c ^ ((r >> 1) & 3)) << 4); };
      auto load_res = [&](int c0, uint4* out4) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int r = m0 + quad * 32 + i * 8 + crow;
          out4[i] = r < rows ? __ldg(reinterpret_cast<const uint4*>(p.residual + static_cast<size_t>(r) * p.ldr + c0) +
                                     cpiece)
                             : make_uint4(0, 0, 0, 0);
        }
      };
      uint4 rc[4];
      load_res(part * 96, rc);
      if (!MLP_TIMED(7, mbar_wait(acc2_full, tile_n & 1, abort_flag, p.err))) break;
      tc_fence_after();
#ifdef BBH_MLP_TRACE
      const long long ln_t0 = clock64();
#endif
      const int row = m0 + rloc;
      float shift = 0.f, s1 = 0.f, s2 = 0.f;
#pragma unroll 1
      for (int ch = 0; ch < 3; ++ch) {
        const int c0 = part * 96 + ch * 32;
        // stage this piece's residual (coalesced rows), fetch the next one
#pragma unroll
        for (int i = 0; i < 4; ++i) *reinterpret_cast<uint4*>(stg_at(i * 8 + crow, cpiece)) = rc[i];
        if (ch < 2) load_res(c0 + 32, rc);
        __syncwarp();
        float v[32];
        tmem_ld32(acc2 + ch * 32, v);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float r8[8];
          unpack_half8(*reinterpret_cast<const uint4*>(stg_at(lane, q)), r8);
#pragma unroll
          for (int e = 0; e < 8; ++e) v[q * 8 + e] += s_b2[c0 + q * 8 + e] + r8[e];
        }
        __syncwarp();  // staging read before the next piece overwrites it
        if (ch == 0) shift = v[0];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float d = v[e] - shift;
          s1 += d;
          s2 += d * d;
        }
        tmem_st32(acc2 + ch * 32, v);  // acc + b2 + residual, read back by the second pass
      }
      // per-part mean and M2 combined over the 4 parts of the row (Chan et al.)
      float* rs = red;
      rs[part * kBM + rloc] = shift + s1 * (1.0f / 96);
      rs[4 * kBM + part * kBM + rloc] = fmaxf(s2 - s1 * s1 * (1.0f / 96), 0.f);
      named_barrier(1 + quad, 128);
      float mean = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) mean += rs[i * kBM + rloc];
      mean *= 0.25f;
      float m2 = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float d = rs[i * kBM + rloc] - mean;
        m2 += rs[4 * kBM + i * kBM + rloc] + d * d * 96;
      }
      const float rstd = rsqrtf(m2 * (1.0f / kHidden) + p.eps);
      named_barrier(1 + quad, 128);  // every part has read the statistics before the next tile
      (void)row;
#pragma unroll 1
      for (int ch = 0; ch < 3; ++ch) {
        const int c0 = part * 96 + ch * 32;
        float v[32];
        tmem_ld32(acc2 + ch * 32, v);
        if (ch == 2) warp_arrive(acc2_free);  // the accumulator has been read
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 g0 = *reinterpret_cast<const float4*>(s_gamma + c0 + q * 8);
          const float4 g1 = *reinterpret_cast<const float4*>(s_gamma + c0 + q * 8 + 4);
          const float4 b0 = *reinterpret_cast<const float4*>(s_beta + c0 + q * 8);
          const float4 b1v = *reinterpret_cast<const float4*>(s_beta + c0 + q * 8 + 4);
          const float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
          const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1v.x, b1v.y, b1v.z, b1v.w};
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            o[e] = pack_half2((v[q * 8 + 2 * e] - mean) * rstd * gg[2 * e] + bb[2 * e],
                              (v[q * 8 + 2 * e + 1] - mean) * rstd * gg[2 * e + 1] + bb[2 * e + 1]);
          *reinterpret_cast<uint4*>(stg_at(lane, q)) = make_uint4(o[0], o[1], o[2], o[3]);
        }
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int r = m0 + quad * 32 + i * 8 + crow;
          if (r < rows)
            reinterpret_cast<uint4*>(p.C + static_cast<size_t>(r) * p.ldc + c0)[cpiece] =
                *reinterpret_cast<const uint4*>(stg_at(i * 8 + crow, cpiece));
        }
        __syncwarp();
      }
#ifdef BBH_MLP_TRACE
      trace_acc[8] += clock64() - ln_t0;
#endif
      ++tile_n;
    }
  }

#ifdef BBH_MLP_TRACE
  if (lane == 0 && warp <= 2)
    for (int i = 0; i < 12; ++i) atomicAdd(&g_mlp_trace[i], static_cast<unsigned long long>(trace_acc[i]));
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
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

// ======================================================================== host side

int make_mlp_plan(MlpPlan* plan, const __half* Y, int rows_cap, const __half* W1, const __half* W2, __half* C,
                  int num_sms) {
  if (!plan || !Y || !W1 || !W2 || !C || rows_cap <= 0) return BBH_ERR_ARG;
  std::memset(plan, 0, sizeof(*plan));
  int rc = encode_2d(&plan->tmX, Y, rows_cap, kHidden, kHidden, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = encode_2d(&plan->tmW1, W1, kFfn, kHidden, kHidden, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = encode_2d(&plan->tmW2, W2, kHidden, kFfn, kFfn, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  const int tiles = (rows_cap + kBM - 1) / kBM;
  plan->grid = tiles < num_sms ? tiles : num_sms;
  plan->p.residual = Y;
  plan->p.ldr = kHidden;
  plan->p.C = C;
  plan->p.ldc = kHidden;
  plan->p.eps = 1e-12f;
  return BBH_OK;
}

cudaError_t launch_mlp(const MlpPlan& plan, cudaStream_t stream, bool pdl) {
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(mlp_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  return launch_ex(mlp_fused_kernel, dim3(plan.grid), dim3(kThreads), kSmem, stream, pdl, 1, plan.tmX, plan.tmW1,
                   plan.tmW2, plan.p);
}

}  // namespace bbh
