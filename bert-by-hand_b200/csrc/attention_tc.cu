// Tensor-core (tcgen05 / TMEM) attention for sentences of at most 128 tokens.
// Replaces the reference's scores -> masked softmax -> context kernels
// (src/kernels/attention.cu:17-121, src/kernels/softmax.cu:26-73) for packed varlen input.
//
// A CTA of 128 threads processes one 128-row tile at a time. The tile packs G "slots" of
// Lp rows (Lp = 16, 32, 64 or 128: the smallest power of two >= L, G = 128 / Lp), one per
// head of the same sentence, so short sentences still fill the MMA rows:
//   1. Q, K, V slices of the fused QKV buffer go to shared memory with cp.async (64-byte
//      swizzled rows of 32 fp16; rows past the sentence are zero-filled), double buffered
//      across tiles.
//   2. One thread issues S = Q K^T (tcgen05.mma, M = N = 128, K = 32) into TMEM.
//   3. Thread t owns query row t (TMEM lane t) and reads the columns of its slot's keys (a
//      key of another head, or past the sentence end, is dropped). Rows of up to 64 keys
//      keep their scores in registers: row max, then exp2-domain exponentials and sum;
//      longer rows walk 32-key chunks once against a reference max raised (with a
//      warp-wide rewrite of the P already written) only when a chunk exceeds it by more
//      than 2^8. P goes as fp16 pairs back into TMEM columns already read (P[k] at column
//      k/2) -- no warp shuffles, no shared-memory or global copy of S or P. Warps whose 32
//      rows hold no query skip.
//   4. One thread issues O = P V (tcgen05.mma with A = P read from TMEM, M = 128, N = 32,
//      K = the keys in use, V as an MN-major shared-memory operand) into columns 64-95;
//      thread t normalises its row by its softmax sum and stores the 32 head dimensions to
//      the merged context [T, 384].
// TMEM 128 columns, 48 KB shared memory and 128 registers per thread: four CTAs per SM.
// A key is also dropped where the token mask is 0 (padded calls), as softmax.cu:43-59 does
// (one bit per key row, built with __ballot_sync when the tile is staged); a row with no
// usable key gives zeros.
#include "common.cuh"
#include "internal.h"

#include <type_traits>

namespace bbh {

constexpr int kTcThreads = 128;
constexpr int kTcRows = 128;
constexpr int kTcCuCache = 1152;  // cu_seqlens entries cached in shared memory

struct TcBuf {  // one tile's operands, each 128 rows x 64 B, 64-byte swizzle
  uint8_t q[kTcRows * 64];
  uint8_t k[kTcRows * 64];
  uint8_t v[kTcRows * 64];
};
static_assert(sizeof(TcBuf) % 1024 == 0, "swizzled operands must stay 1024-byte aligned");

struct TcSmem {
  TcBuf buf[2];
  uint32_t keybits[2][kTcRows / 32];  // bit r: key row r usable (padded calls with a token mask)
  uint64_t bar_s, bar_o;
  uint32_t tmem;
  int abort_flag;
  int cu[1];  // cached cu_seqlens follow (variable length)
};

// K-major operand with 64-byte rows (32 fp16) and 64-byte swizzle: SBO = 8 rows x 64 B.
__device__ __forceinline__ uint64_t sw64_kmajor_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr & 0x3FFFF) >> 4);
  d |= static_cast<uint64_t>(1) << 16;         // LBO (unused for swizzled K-major)
  d |= static_cast<uint64_t>(512 >> 4) << 32;  // SBO
  d |= static_cast<uint64_t>(1) << 46;         // sm_100 descriptor version
  d |= static_cast<uint64_t>(4) << 61;         // SWIZZLE_64B
  return d;
}

// MN-major operand (V: rows = keys = K dimension, 32 fp16 of N per 64-byte row), 64-byte
// swizzle: 8 K-rows per 512-byte atom (SBO); one 32-element N group, so LBO is not used.
__device__ __forceinline__ uint64_t sw64_mnmajor_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr & 0x3FFFF) >> 4);
  d |= static_cast<uint64_t>(4096 >> 4) << 16;  // LBO: next 32-wide N group (never used, N = 32)
  d |= static_cast<uint64_t>(512 >> 4) << 32;   // SBO: next 8 K-rows
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(4) << 61;
  return d;
}

__device__ __forceinline__ void cp_async16_tc(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit_tc() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_tc() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// log2 of the slot height for a sentence of `len` tokens
__device__ __forceinline__ int slot_log2(int len) { return len <= 16 ? 4 : len <= 32 ? 5 : len <= 64 ? 6 : 7; }

// Items are enumerated head-major, item = h * batch + b: with a grid-stride walk every CTA
// then meets a mix of sentences and heads. (Sentence-major order aliases with the stride:
// the packed-head items, h % G == 0, would all land on a quarter of the CTAs.)
struct TcItem {
  int item;  // h0 * batch + b, or -1
  int h0, start, len;
};

__device__ __forceinline__ TcItem tc_find(const int* cu, int batch, int item, int step, int items) {
  TcItem u;
  for (; item < items; item += step) {
    const int b = item % batch;
    const int h = item / batch;
    const int start = cu[b];
    const int len = cu[b + 1] - start;
    if (len <= 0 || len > kTcRows) continue;
    const int G = kTcRows >> slot_log2(len);
    if (h % G) continue;
    u.item = item;
    u.h0 = h;
    u.start = start;
    u.len = len;
    return u;
  }
  u.item = -1;
  return u;
}

__device__ __forceinline__ void tc_load(const AttnParams& p, const uint8_t* tokmask, const TcItem& u, TcBuf& B,
                                        uint32_t* keybits, int tid) {
  const int lg = slot_log2(u.len);
  const int G = kTcRows >> lg;
  const int h0 = u.h0;
  const int nh = (kHeads - h0) < G ? (kHeads - h0) : G;
  const __half* base = p.qkv + static_cast<size_t>(u.start) * kQkvLd + h0 * kHeadDim;
  const uint32_t sq = smem_u32(B.q), sk = smem_u32(B.k), sv = smem_u32(B.v);
  // 128 rows x 4 pieces per operand; thread tid handles piece (tid & 3) of rows tid/4 + 32 i
  const int c = tid & 3;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = (tid >> 2) + 32 * i;
    const int s = r >> lg, q = r & ((1 << lg) - 1);
    const bool ok = s < nh && q < u.len;
    const __half* src = base + static_cast<size_t>(ok ? q : 0) * kQkvLd + s * kHeadDim + c * 8;
    const uint32_t off = r * 64 + ((c ^ ((r >> 1) & 3)) << 4);
    cp_async16_tc(sq + off, src, ok ? 16 : 0);
    cp_async16_tc(sk + off, src + kHidden, ok ? 16 : 0);
    cp_async16_tc(sv + off, src + 2 * kHidden, ok ? 16 : 0);
  }
  if (tokmask) {
    // one bit per key row, a word per warp (row r = thread r)
    const int r = tid;
    const int s = r >> lg, q = r & ((1 << lg) - 1);
    const uint32_t word = __ballot_sync(0xffffffffu, s < nh && q < u.len && tokmask[u.start + q] != 0);
    if ((r & 31) == 0) keybits[r >> 5] = word;
  }
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&w)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7]), "r"(w[8]), "r"(w[9]),
      "r"(w[10]), "r"(w[11]), "r"(w[12]), "r"(w[13]), "r"(w[14]), "r"(w[15])
      : "memory");
}
// 32 lanes x 16 columns -> 16 registers per thread
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st8_zero(uint32_t taddr) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1};" ::"r"(taddr), "r"(0)
               : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// D[tmem] (+)= A[tmem] * B[smem]: A (K-major fp16 pairs, 8 columns per K=16 step) read
// from tensor memory.
__device__ __forceinline__ void tc_mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__global__ void __launch_bounds__(kTcThreads, 4) attention_tc_kernel(AttnParams p) {
  extern __shared__ uint8_t tc_raw[];
  TcSmem& sm = *reinterpret_cast<TcSmem*>((reinterpret_cast<uintptr_t>(tc_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x;
  pdl_launch_dependents();
  pdl_wait();  // Q/K/V and the sentence table come from the previous kernels
  const int warp = tid >> 5;

  const int batch = p.meta ? p.meta[0] : p.batch;
  const uint8_t* tokmask = (p.meta && p.meta[3] == 0) ? nullptr : p.tokmask;
  const int items = batch * kHeads;
  const int* cu = p.cu;
  if (batch < kTcCuCache) {
    for (int i = tid; i <= batch; i += kTcThreads) sm.cu[i] = p.cu[i];
    cu = sm.cu;
  }
  if (tid == 0) {
    mbar_init(&sm.bar_s, 1);
    mbar_init(&sm.bar_o, 1);
    sm.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(&sm.tmem, 128);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem;  // S: columns [0, 128); P (fp16 pairs) [0, 64); O [64, 96)
  const uint32_t t_o = tmem + 64;
  const int row = tid;
  const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
  volatile int* abort_flag = &sm.abort_flag;

  constexpr uint32_t idesc_s = idesc_f16_f32(128, 128);              // Q K^T, both K-major
  constexpr uint32_t idesc_o = idesc_f16_f32(128, 32) | (1u << 16);  // P V, B (V) MN-major

  TcItem cur = tc_find(cu, batch, blockIdx.x, gridDim.x, items);
  int bi = 0;
  uint32_t ph = 0;
  if (cur.item >= 0) {
    tc_load(p, tokmask, cur, sm.buf[0], sm.keybits[0], tid);
    cp_async_commit_tc();
  }
  while (cur.item >= 0) {
    const TcItem nxt = tc_find(cu, batch, cur.item + gridDim.x, gridDim.x, items);
    if (nxt.item >= 0) {
      tc_load(p, tokmask, nxt, sm.buf[bi ^ 1], sm.keybits[bi ^ 1], tid);
      cp_async_commit_tc();
      cp_async_wait_tc<1>();
    } else {
      cp_async_wait_tc<0>();
    }
    fence_async_shared();  // this thread's cp.async data -> visible to the tensor core
    __syncthreads();
    TcBuf& B = sm.buf[bi];
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int k = 0; k < 2; ++k)
        tc_mma_f16(tmem, sw64_kmajor_desc(smem_u32(B.q) + k * 32), sw64_kmajor_desc(smem_u32(B.k) + k * 32),
                   idesc_s, k);
      tc_commit(&sm.bar_s);
    }

    // ---- geometry of this tile (all warp-uniform except slot/q/row_ok)
    const int len = cur.len;
    const int lg = slot_log2(len);
    const int Lp = 1 << lg;
    const int G = kTcRows >> lg;
    const int h0 = cur.h0;
    const int nh = (kHeads - h0) < G ? (kHeads - h0) : G;
    const int slot = row >> lg, q = row & (Lp - 1);
    const bool row_ok = slot < nh && q < len;
    const int s0 = (warp * 32) >> lg;  // slot of this warp's first row
    const bool warp_active = Lp <= 16 ? (s0 < nh) : (s0 < nh && ((warp * 32) & (Lp - 1)) < len);
    // TMEM columns of the warp's rows' slot keys, in 32-column chunks
    const int c_lo = Lp <= 32 ? warp * 32 : s0 * Lp;
    const int nchunk = Lp <= 32 ? 1 : (len + 31) >> 5;
    const int off = slot * Lp - c_lo;  // my keys start at this column of the warp's range
    // keys the O MMA contracts over
    const int kused = Lp == kTcRows ? ((len + 15) & ~15) : nh * Lp;

    if (!mbar_wait(&sm.bar_s, ph, abort_flag, nullptr)) break;
    tc_fence_after();
    const float scale = p.scale_log2;
    // Usable keys of chunk ch as a bit mask over its 32 columns: this row's keys are the
    // columns [off, off + len) of the warp's range, further limited by the token mask.
    auto chunk_mask = [&](int ch) -> uint32_t {
      const int lo = max(off - ch * 32, 0), hi = min(off - ch * 32 + len, 32);
      uint32_t m = 0;
      if (hi > lo) m = (hi >= 32 ? 0xffffffffu : ((1u << hi) - 1u)) & ~((1u << lo) - 1u);
      if (tokmask) m &= sm.keybits[bi][(c_lo + ch * 32) >> 5];  // chunks start on 32-row words
      return row_ok ? m : 0u;
    };
    float sum = 0.f;
    // One or two 32-key chunks (sentences of <= 64 tokens): the row's scores stay in
    // registers between the max and the exponentials (one TMEM read), masked scores are
    // set to -inf so that their 2^(...) is 0 without a second select.
    auto short_row = [&](auto nc_tag) {
      constexpr int NC = decltype(nc_tag)::value;
      const uint32_t trow = tmem + lane_off;
      float t[NC][32];
      uint32_t m[NC];
#pragma unroll
      for (int c = 0; c < NC; ++c) m[c] = chunk_mask(c);
      if constexpr (NC == 1) {
        tmem_ld32(trow + c_lo, t[0]);
      } else {
        float t64[64];
        tmem_ld64(trow + c_lo, trow + c_lo + 32, t64);
#pragma unroll
        for (int j = 0; j < 32; ++j) t[0][j] = t64[j], t[1][j] = t64[32 + j];
      }
      float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        if (m[c] != 0xffffffffu) {
#pragma unroll
          for (int j = 0; j < 32; ++j) t[c][j] = (m[c] >> j) & 1u ? t[c][j] : -INFINITY;
        }
#pragma unroll
        for (int j = 0; j < 32; j += 2) mq[(j >> 1) & 3] = fmax3(mq[(j >> 1) & 3], t[c][j], t[c][j + 1]);
      }
      const float mx = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3]));
      const float msc = mx == -INFINITY ? 0.f : mx * scale;
      float sq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        uint32_t w[16];
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          float e0, e1;
          asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e0) : "f"(fmaf(t[c][j], scale, -msc)));
          asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e1) : "f"(fmaf(t[c][j + 1], scale, -msc)));
          sq[j & 3] += e0;
          sq[(j + 1) & 3] += e1;
          w[j >> 1] = pack_half2(e0, e1);
        }
        tmem_st16(trow + (c_lo >> 1) + c * 16, w);
      }
      sum = (sq[0] + sq[1]) + (sq[2] + sq[3]);
      const int z_lo = c_lo >> 4, z_hi = z_lo + NC * 2, z_used = kused >> 4;
#pragma unroll 1
      for (int z = 0; z < z_used; ++z)
        if (z < z_lo || z >= z_hi) tmem_st8_zero(trow + z * 8);
      tmem_wait_st();
    };
    if (warp_active && nchunk == 1) {
      short_row(std::integral_constant<int, 1>{});
    } else if (warp_active && nchunk == 2) {
      short_row(std::integral_constant<int, 2>{});
    } else if (warp_active) {
      // Three or four chunks: one pass with a lazily raised reference (as in the long
      // kernel): the first chunk's max is the reference m; a later chunk whose max exceeds
      // it by more than 2^8 raises it and rescales the P already written (this row's own
      // TMEM lane) and the partial sums, so P stays <= 256 in fp16. P of chunk ch goes to
      // columns 16 ch .. +16, over S columns already read.
      const uint32_t trow = tmem + lane_off;
      constexpr float kRaise = 8.f;
      float mref = -INFINITY;
      float sq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
      for (int ch = 0; ch < nchunk; ++ch) {
        const uint32_t m = chunk_mask(ch);
        float t[32];
        tmem_ld32(trow + c_lo + ch * 32, t);
        if (m != 0xffffffffu) {
#pragma unroll
          for (int j = 0; j < 32; ++j) t[j] = (m >> j) & 1u ? t[j] : -INFINITY;
        }
        float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int j = 0; j < 32; j += 2) mq[(j >> 1) & 3] = fmax3(mq[(j >> 1) & 3], t[j], t[j + 1]);
        const float cmax = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3]));
        float alpha = 1.f;
        if (cmax != -INFINITY && (mref == -INFINITY || (cmax - mref) * scale > kRaise)) {
          if (mref != -INFINITY) {
            alpha = exp2f((mref - cmax) * scale);
#pragma unroll
            for (int k = 0; k < 4; ++k) sq[k] *= alpha;
          }
          mref = cmax;
        }
        // TMEM loads and stores are warp-collective: the whole warp rewrites its earlier P
        // when any of its rows raised (alpha 1 leaves a row unchanged)
        if (ch > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
          tmem_wait_st();  // this warp's earlier P stores, read back below
#pragma unroll 1
          for (int c = 0; c < ch; ++c) {
            float pv[16];
            tmem_ld16(trow + (c_lo >> 1) + c * 16, pv);
            uint32_t w[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {  // fp32 alpha, one rounding back to fp16
              const uint32_t u = __float_as_uint(pv[i]);
              const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u));
              w[i] = pack_half2(f.x * alpha, f.y * alpha);
            }
            tmem_st16(trow + (c_lo >> 1) + c * 16, w);
          }
        }
        const float msc = mref == -INFINITY ? 0.f : mref * scale;
        uint32_t w[16];
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          float e0, e1;
          asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e0) : "f"(fmaf(t[j], scale, -msc)));
          asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e1) : "f"(fmaf(t[j + 1], scale, -msc)));
          sq[j & 3] += e0;
          sq[(j + 1) & 3] += e1;
          w[j >> 1] = pack_half2(e0, e1);
        }
        tmem_st16(trow + (c_lo >> 1) + ch * 16, w);
      }
      sum = (sq[0] + sq[1]) + (sq[2] + sq[3]);
      // zeros in the P columns the O MMA reads outside this warp's key range (8 columns =
      // 16 keys at a time; only this warp's own lanes are written)
      const int z_lo = c_lo >> 4, z_hi = z_lo + nchunk * 2, z_used = kused >> 4;
#pragma unroll 1
      for (int z = 0; z < z_used; ++z)
        if (z < z_lo || z >= z_hi) tmem_st8_zero(trow + z * 8);
      tmem_wait_st();
    }
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      for (int k = 0; k < (kused >> 4); ++k) {
        const uint64_t bdesc = sw64_mnmajor_desc(smem_u32(B.v) + k * 1024);
        tc_mma_f16_ts(t_o, tmem + k * 8, bdesc, idesc_o, k);
      }
      tc_commit(&sm.bar_o);
    }
    if (!mbar_wait(&sm.bar_o, ph, abort_flag, nullptr)) break;
    tc_fence_after();
    if (warp_active) {
      float o[32];
      tmem_ld32(t_o + lane_off, o);
      if (row_ok) {
        const float inv = sum > 0.f ? 1.0f / sum : 0.f;
        __half* out = p.ctx + static_cast<size_t>(cur.start + q) * kHidden + (h0 + slot) * kHeadDim;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint4 w;
          uint32_t* ww = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
          for (int e = 0; e < 4; ++e) ww[e] = pack_half2(o[j * 8 + 2 * e] * inv, o[j * 8 + 2 * e + 1] * inv);
          *reinterpret_cast<uint4*>(out + j * 8) = w;
        }
      }
    }
    tc_fence_before();
    ph ^= 1;
    bi ^= 1;
    cur = nxt;
  }
  cp_async_wait_tc<0>();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

// ======================================================================== long sentences
// Sentences of 129-512 tokens (the reference caps seq at 128; configs[4] runs 512): one CTA
// item is (sentence, head, block of 128 query rows). Q of the block and all of the head's
// K and V go to shared memory once (cp.async, 64-byte swizzle, zero-filled past the end);
// the keys are then walked in blocks of 64 with the online softmax of flash attention:
//   S_j = Q K_j^T (tcgen05, M = 128, N = 64) into one of two TMEM buffers, so the S-MMA of
//   block j + 2 is queued behind the P.V-MMA of block j and overlaps the softmax of j + 1;
//   thread t (query row t) keeps a reference max m and the sum l, and writes
//   P_j = 2^(s*scale - m*scale) as fp16 pairs into one of two P buffers. The reference is
//   raised (and l and the row of O in TMEM rescaled) only when a block's max exceeds it by
//   more than 2^8, so P stays <= 256 and most blocks need no rescale: then the P.V-MMA of
//   block j is issued without waiting for the one of block j - 1. When some row does need
//   it, the CTA waits once for the issued MMAs and rescales;
//   O += P_j V_j (tcgen05, A = P from TMEM, V MN-major in shared memory).
// Two threads per query row: warps w and w + 4 share TMEM lane quadrant w; both read the
// whole 64-key block for its row max (no exchange), then each takes 32 of its keys (the
// two partial sums meet in shared memory once per item). One CTA barrier per block (before
// the P.V issue), two when some row raises its reference.
// TMEM: S buffers at columns [0, 64) and [64, 128), O at [128, 160), P buffers (fp16
// pairs, 32 columns per block) at [160, 192) and [192, 224) (256 allocated);
// ~80 KB of shared memory: two CTAs (16 warps) per SM.
constexpr int kLongThreads = 256;
constexpr int kLongMax = 512;  // keys per sentence
constexpr int kKeyBlk = 64;

struct LongSmem {
  uint8_t q[kTcRows * 64];
  uint8_t k[kLongMax * 64];
  uint8_t v[kLongMax * 64];
  uint32_t keybits[kLongMax / 32];  // bit k: key k usable (padded calls with a token mask)
  float part[2][kTcRows];  // per-half partial row max, then partial row sum
  uint64_t bar_s[2], bar_o, bar_fix;
  uint32_t tmem;
  int abort_flag;
  int cu[1];  // cached cu_seqlens follow
};

struct LongItem {
  int item, h, qb, start, len;
};

// items are (head, sentence, query block), head-major like the short kernel
__device__ __forceinline__ LongItem long_find(const int* cu, int batch, int item, int step, int items, int min_len) {
  LongItem u;
  for (; item < items; item += step) {
    const int qb = item & 3;
    const int rest = item >> 2;
    const int b = rest % batch;
    const int h = rest / batch;
    const int start = cu[b];
    const int len = cu[b + 1] - start;
    if (len < min_len || len > kLongMax || qb * kTcRows >= len) continue;
    u.item = item;
    u.h = h;
    u.qb = qb;
    u.start = start;
    u.len = len;
    return u;
  }
  u.item = -1;
  return u;
}

__global__ void __launch_bounds__(kLongThreads, 2) attention_long_kernel(AttnParams p) {
  extern __shared__ uint8_t lg_raw[];
  LongSmem& sm = *reinterpret_cast<LongSmem*>((reinterpret_cast<uintptr_t>(lg_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x;
  pdl_launch_dependents();
  pdl_wait();
  const int warp = tid >> 5;
  const int batch = p.meta ? p.meta[0] : p.batch;
  const uint8_t* tokmask = (p.meta && p.meta[3] == 0) ? nullptr : p.tokmask;
  const int items = batch * kHeads * 4;
  const int* cu = p.cu;
  if (batch < kTcCuCache) {
    for (int i = tid; i <= batch; i += kLongThreads) sm.cu[i] = p.cu[i];
    cu = sm.cu;
  }
  if (tid == 0) {
    mbar_init(&sm.bar_s[0], 1);
    mbar_init(&sm.bar_s[1], 1);
    mbar_init(&sm.bar_o, 1);
    mbar_init(&sm.bar_fix, 1);
    sm.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(&sm.tmem, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem;
  const uint32_t t_o = tmem + 128;
  const uint32_t t_p = tmem + 160;  // P of block j in buffer j & 1: never over unread S columns
  const int quad = warp & 3, half = warp >> 2;  // TMEM lane quadrant; key half of a block
  const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
  volatile int* abort_flag = &sm.abort_flag;
  constexpr uint32_t idesc_s = idesc_f16_f32(128, kKeyBlk);            // Q K^T, both K-major
  constexpr uint32_t idesc_o = idesc_f16_f32(128, 32) | (1u << 16);    // P V, V MN-major
  const float scale = p.scale_log2;
  uint32_t ph_s = 0, ph_o = 0, ph_fix = 0;  // ph_s bit b: phase of bar_s[b]
  constexpr float kRescaleLog2 = 8.f;  // raise the reference max when a block exceeds it by 2^8

  for (LongItem u = long_find(cu, batch, blockIdx.x, gridDim.x, items, p.min_len); u.item >= 0;
       u = long_find(cu, batch, u.item + gridDim.x, gridDim.x, items, p.min_len)) {
    const int len = u.len;
    const int nkb = (len + kKeyBlk - 1) / kKeyBlk;
    const int q0 = u.qb * kTcRows;
    // ---- stage Q (128 rows), K and V (nkb * 64 rows) of this head
    {
      const __half* base = p.qkv + static_cast<size_t>(u.start) * kQkvLd + u.h * kHeadDim;
      const uint32_t sq = smem_u32(sm.q), sk = smem_u32(sm.k), sv = smem_u32(sm.v);
      const int c = tid & 3;
      for (int r = tid >> 2; r < kTcRows; r += kLongThreads / 4) {
        const bool ok = q0 + r < len;
        const uint32_t off = r * 64 + ((c ^ ((r >> 1) & 3)) << 4);
        cp_async16_tc(sq + off, base + static_cast<size_t>(ok ? q0 + r : 0) * kQkvLd + c * 8, ok ? 16 : 0);
      }
      for (int r = tid >> 2; r < nkb * kKeyBlk; r += kLongThreads / 4) {
        const bool ok = r < len;
        const uint32_t off = r * 64 + ((c ^ ((r >> 1) & 3)) << 4);
        const __half* src = base + static_cast<size_t>(ok ? r : 0) * kQkvLd + c * 8;
        cp_async16_tc(sk + off, src + kHidden, ok ? 16 : 0);
        cp_async16_tc(sv + off, src + 2 * kHidden, ok ? 16 : 0);
      }
      if (tokmask)  // one bit per key, a word per warp and pass (warp-uniform loop)
        for (int r = tid; r < nkb * kKeyBlk; r += kLongThreads) {
          const uint32_t word = __ballot_sync(0xffffffffu, r < len && tokmask[u.start + r] != 0);
          if ((r & 31) == 0) sm.keybits[r >> 5] = word;
        }
      cp_async_commit_tc();
      cp_async_wait_tc<0>();
      fence_async_shared();
      __syncthreads();
    }
    auto issue_s = [&](int j) {
      const int b = j & 1;
#pragma unroll
      for (int kk = 0; kk < 2; ++kk)
        tc_mma_f16(tmem + b * kKeyBlk, sw64_kmajor_desc(smem_u32(sm.q) + kk * 32),
                   sw64_kmajor_desc(smem_u32(sm.k) + j * kKeyBlk * 64 + kk * 32), idesc_s, kk);
      tc_commit(&sm.bar_s[b]);
    };
    if (tid == 0) {
      tc_fence_after();
      issue_s(0);
      if (nkb > 1) issue_s(1);
    }
    const int row = quad * 32 + (tid & 31);
    const bool row_ok = q0 + row < len;
    float m = -INFINITY, l = 0.f;
    bool failed = false;
    for (int j = 0; j < nkb; ++j) {
      const int b = j & 1;
      if (!mbar_wait(&sm.bar_s[b], (ph_s >> b) & 1u, abort_flag, nullptr)) {
        failed = true;
        break;
      }
      ph_s ^= 1u << b;
      tc_fence_after();
      // usable keys of a 32-key half of this block: k < len (and the token mask), for a
      // valid query row
      auto half_mask = [&](int hh) -> uint32_t {
        const int k0 = j * kKeyBlk + hh * 32;
        const int n_ok = min(max(len - k0, 0), 32);
        uint32_t mm = n_ok >= 32 ? 0xffffffffu : ((1u << n_ok) - 1u);
        if (tokmask) mm &= sm.keybits[k0 >> 5];
        return row_ok ? mm : 0u;
      };
      // the block's row max: each of the row's two threads reads both halves (no exchange)
      float bmax;
      {
        float t2[32];
        tmem_ld32(tmem + lane_off + b * kKeyBlk + (half ^ 1) * 32, t2);
        const uint32_t mk2 = half_mask(half ^ 1);
        if (mk2 != 0xffffffffu) {
#pragma unroll
          for (int e = 0; e < 32; ++e) t2[e] = (mk2 >> e) & 1u ? t2[e] : -INFINITY;
        }
        float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int e = 0; e < 32; e += 2) mq[(e >> 1) & 3] = fmax3(mq[(e >> 1) & 3], t2[e], t2[e + 1]);
        bmax = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3]));
      }
      float t[32];
      tmem_ld32(tmem + lane_off + b * kKeyBlk + half * 32, t);
      const uint32_t mk = half_mask(half);
      if (mk != 0xffffffffu) {
#pragma unroll
        for (int e = 0; e < 32; ++e) t[e] = (mk >> e) & 1u ? t[e] : -INFINITY;
      }
      {
        float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int e = 0; e < 32; e += 2) mq[(e >> 1) & 3] = fmax3(mq[(e >> 1) & 3], t[e], t[e + 1]);
        bmax = fmaxf(bmax, fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3])));
      }
      // raise the reference max if this block exceeds it by more than 2^8 (always for the
      // first usable block); alpha rescales what was accumulated against the old reference
      float alpha = 1.f;
      const bool raise = bmax != -INFINITY && (m == -INFINITY || (bmax - m) * scale > kRescaleLog2);
      if (raise) {
        alpha = m == -INFINITY ? 0.f : exp2f((m - bmax) * scale);
        l *= alpha;
        m = bmax;
      }
      const float msc = m == -INFINITY ? 0.f : m * scale;
      float bsum = 0.f;
      {
        uint32_t w[16];
        // masked keys already hold -inf, so 2^(-inf) = 0 there: no per-key select
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float e0, e1;
          asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e0) : "f"(fmaf(t[e], scale, -msc)));
          asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e1) : "f"(fmaf(t[e + 1], scale, -msc)));
          bsum += e0 + e1;
          w[e >> 1] = pack_half2(e0, e1);
        }
        tmem_st16(t_p + lane_off + b * 32 + half * 16, w);  // P pairs: key k at column k / 2
      }
      l += bsum;  // this half's share of the row sum (both halves use the same reference m)
      tmem_wait_st();
      tc_fence_before();
      // one barrier per block: P of every row is written; when some row raised its reference,
      // O (earlier blocks' P.V) is rescaled first, once the issued MMAs have landed
      if (__syncthreads_or(raise && j > 0 && alpha != 1.f)) {
        if (tid == 0) tc_commit(&sm.bar_fix);  // arrives when every MMA issued so far is done
        if (!mbar_wait(&sm.bar_fix, ph_fix, abort_flag, nullptr)) {
          failed = true;
          break;
        }
        ph_fix ^= 1;
        tc_fence_after();
        if (half == 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
          float o[32];
          tmem_ld32(t_o + lane_off, o);
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] *= alpha;
          tmem_st32(t_o + lane_off, o);
        }
        tc_fence_before();
        __syncthreads();
      }
      if (tid == 0) {
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < kKeyBlk / 16; ++k)
          tc_mma_f16_ts(t_o, t_p + b * 32 + k * 8,
                        sw64_mnmajor_desc(smem_u32(sm.v) + (j * (kKeyBlk / 16) + k) * 1024), idesc_o,
                        (j > 0 || k > 0) ? 1u : 0u);
        if (j + 1 == nkb) tc_commit(&sm.bar_o);  // the item's last P.V
        if (j + 2 < nkb) issue_s(j + 2);        // queued behind this P.V, which reads the buffer
      }
    }
    if (failed) break;
    sm.part[half][row] = l;
    __syncthreads();
    const float l_row = l + sm.part[half ^ 1][row];
    if (!mbar_wait(&sm.bar_o, ph_o, abort_flag, nullptr)) break;
    ph_o ^= 1;
    tc_fence_after();
    {
      float o[16];  // this half's 16 of the row's 32 output dimensions
      tmem_ld16(t_o + lane_off + half * 16, o);
      if (row_ok) {
        const float inv = l_row > 0.f ? 1.0f / l_row : 0.f;
        __half* out = p.ctx + static_cast<size_t>(u.start + q0 + row) * kHidden + u.h * kHeadDim + half * 16;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          uint4 wv;
          uint32_t* ww = reinterpret_cast<uint32_t*>(&wv);
#pragma unroll
          for (int e = 0; e < 4; ++e) ww[e] = pack_half2(o[j * 8 + 2 * e] * inv, o[j * 8 + 2 * e + 1] * inv);
          *reinterpret_cast<uint4*>(out + j * 8) = wv;
        }
      }
    }
    tc_fence_before();
    __syncthreads();  // shared memory and TMEM free for the next item
  }
  cp_async_wait_tc<0>();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

int attention_long_smem() { return static_cast<int>(sizeof(LongSmem)) + 4 * kTcCuCache + 1024; }

cudaError_t launch_attention_long(const AttnParams& p, int grid, cudaStream_t stream, bool pdl) {
  const int smem = attention_long_smem();
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attention_long_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  return launch_ex(attention_long_kernel, dim3(grid), dim3(kLongThreads), smem, stream, pdl, 1, p);
}

int attention_tc_smem() { return static_cast<int>(sizeof(TcSmem)) + 4 * kTcCuCache + 1024; }

cudaError_t launch_attention_tc(const AttnParams& p, int grid, cudaStream_t stream, bool pdl) {
  const int smem = attention_tc_smem();
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  return launch_ex(attention_tc_kernel, dim3(grid), dim3(kTcThreads), smem, stream, pdl, 1, p);
}

}  // namespace bbh
