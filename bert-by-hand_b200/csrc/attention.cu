// Variable-length (cu_seqlens-packed) multi-head self-attention with online softmax.
// Replaces the reference's three-kernel attention (scores -> masked softmax -> context:
// src/kernels/attention.cu:17-121, src/kernels/softmax.cu:26-73, wired at
// src/model/encoder.cu:37-45), with no S x S buffer and no padding.
//
// Q, K and V are read as strided slices of the fused QKV buffer [T, 1152] (head h at
// columns h*32, 384 + h*32, 768 + h*32), and the context is written straight into the
// merged-heads layout [T, 384], as the reference does.
//
// Work item = (sentence, head, 64-query chunk). A 4-warp CTA owns one item at a time;
// each warp owns 16 query rows. Short sentences pack heads: for L <= 16 the four warps
// take four heads, for L <= 32 two heads with two warps each, so no warp idles on a
// padded query block. Keys are processed in blocks of up to 128 per head. The next
// block's Q/K/V slices are fetched with cp.async (zero-filled past the sentence end)
// into the second of two shared-memory buffers while the current block is computed.
// Scores and P.V use mma.sync m16n8k16 (fp16 in, fp32 accumulate); only the 8-key
// tiles inside the sentence are computed. Softmax runs in fp32 in the exp2 domain with a
// running max and sum per row. A key is dropped when it lies past the sentence end or its
// mask entry is 0 (src/kernels/softmax.cu:43-59); a row whose keys are all masked gives
// zeros, as the reference's softmax does.
#include "common.cuh"
#include "internal.h"

namespace bbh {

constexpr int kAttnThreads = 128;
constexpr int kQRows = 64;     // query rows per CTA item
constexpr int kKeyBlock = 128; // key rows per CTA buffer (all head slots together)
constexpr int kRowPad = 40;    // fp16 per smem row: 80 B keeps ldmatrix rows conflict-free

struct AttnBuf {
  __half q[kKeyBlock][kRowPad];  // up to 128 query rows (whole-sentence items)
  __half k[kKeyBlock][kRowPad];
  __half v[kKeyBlock][kRowPad];
  float bias[kKeyBlock];  // 0 for a usable key, -inf for a dropped one
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// 16-byte async copy; src_bytes == 0 writes zeros without reading.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

constexpr int kCuCache = 1152;  // cu_seqlens entries cached in shared memory (batch <= 1151)

// Heads packed in one CTA item: 4 (L <= 16), 2 (L <= 32) or 1.
__device__ __forceinline__ int heads_per_cta(int len) { return len <= 16 ? 4 : (len <= 32 ? 2 : 1); }

// Work decomposition. item = (b * kHeads + h) << qshift | qc.
//  * max_len <= 128: qshift = 0, one item per (sentence, head) -- or per group of 2/4
//    heads for short sentences; the item's keys fit one buffer and each warp walks its
//    16-row query blocks (w, w+4, ...) against them.
//  * max_len > 128: qc = 64-row query chunk; keys stream through the buffers in blocks
//    of 128 (`kb`), with the softmax state carried across blocks.
struct Unit {
  int item;  // -1 = none
  int kb;
  int start, len;
};

struct Decomp {
  int qshift;  // log2(query chunks per head); 0 = whole sentence per item
  int items;
  __device__ __forceinline__ int qc(int item) const { return item & ((1 << qshift) - 1); }
  __device__ __forceinline__ int h(int item) const { return (item >> qshift) % kHeads; }
  __device__ __forceinline__ int b(int item) const { return (item >> qshift) / kHeads; }
  __device__ __forceinline__ bool streamed() const { return qshift > 0; }
};

__device__ __forceinline__ Unit find_unit(const int* cu, const Decomp& d, int item, int step, int min_len) {
  Unit u;
  for (; item < d.items; item += step) {
    const int qc = d.qc(item);
    const int h = d.h(item);
    const int b = d.b(item);
    const int start = cu[b];
    const int len = cu[b + 1] - start;
    if (len < min_len) continue;
    bool active;
    if (d.streamed()) {
      active = qc * kQRows < len && (len > kKeyBlock || qc == 0) && (heads_per_cta(len) == 1 || h % heads_per_cta(len) == 0);
    } else {
      active = len > 0 && h % heads_per_cta(len) == 0;
    }
    if (active) {
      u.item = item;
      u.kb = 0;
      u.start = start;
      u.len = len;
      return u;
    }
  }
  u.item = -1;
  return u;
}

__device__ __forceinline__ Unit next_unit(const int* cu, const Decomp& d, const Unit& u, int step, int min_len) {
  if (u.item < 0) return u;
  if (u.len > kKeyBlock && (u.kb + 1) * kKeyBlock < u.len) {
    Unit n = u;
    n.kb = u.kb + 1;
    return n;
  }
  return find_unit(cu, d, u.item + step, step, min_len);
}

// Number of query rows an item covers (from q0).
__device__ __forceinline__ int item_qrows(const Unit& u, int q0) {
  if (u.len > kKeyBlock) return u.len - q0 < kQRows ? u.len - q0 : kQRows;
  return u.len;  // whole sentence (<= 128 rows)
}

// Issue the cp.async copies of unit u into buffer `buf` (division-free index math).
__device__ __forceinline__ void load_unit(const AttnParams& p, const uint8_t* tokmask, const Decomp& d, const Unit& u,
                                          AttnBuf& buf, int tid) {
  const int hpc = heads_per_cta(u.len);
  const int kslot = kKeyBlock / hpc;  // key rows per head slot
  const int k0 = u.kb * kKeyBlock;
  const int q0 = d.qc(u.item) * kQRows;
  int krows = u.len - k0;
  krows = krows > kslot ? kslot : krows;
  const int krows16 = (krows + 15) & ~15;
  const int qrows = item_qrows(u, q0);
  const int qrows16 = (qrows + 15) & ~15;
  const int qslot = hpc == 1 ? kKeyBlock : kQRows / hpc;  // query rows per head slot in buf.q
  const __half* base = p.qkv + static_cast<size_t>(u.start) * kQkvLd + d.h(u.item) * kHeadDim;
  const int piece = tid & 3;
  const int r0 = tid >> 2;  // 0..31
  for (int s = 0; s < hpc; ++s) {
    const __half* sb = base + s * kHeadDim + piece * 8;
    for (int r = r0; r < krows16; r += 32) {
      const bool ok = r < krows;
      const __half* src = sb + static_cast<size_t>(ok ? k0 + r : 0) * kQkvLd;
      cp_async16(&buf.k[s * kslot + r][piece * 8], src + kHidden, ok ? 16 : 0);
      cp_async16(&buf.v[s * kslot + r][piece * 8], src + 2 * kHidden, ok ? 16 : 0);
    }
    if (u.kb == 0) {
      for (int r = r0; r < qrows16; r += 32) {
        const bool ok = r < qrows;
        const __half* src = sb + static_cast<size_t>(ok ? q0 + r : 0) * kQkvLd;
        cp_async16(&buf.q[s * qslot + r][piece * 8], src, ok ? 16 : 0);
      }
    }
  }
  if (tid < kKeyBlock) {
    const int j = k0 + tid;
    buf.bias[tid] = (j < u.len && (!tokmask || tokmask[u.start + j])) ? 0.f : -INFINITY;
  }
}

struct SoftmaxState {
  uint32_t qa[2][4];
  float o[4][4];
  float m0, m1, l0, l1;
};

__device__ __forceinline__ void state_begin(SoftmaxState& st, const AttnBuf& B, int qrow, int lane) {
#pragma unroll
  for (int kc = 0; kc < 2; ++kc) {
    const int mi = lane >> 3;
    const int r = qrow + (lane & 7) + (mi & 1) * 8;
    const int c = kc * 16 + (mi >> 1) * 8;
    ldsm_x4(smem_u32(&B.q[r][c]), st.qa[kc][0], st.qa[kc][1], st.qa[kc][2], st.qa[kc][3]);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) st.o[i][j] = 0.f;
  st.m0 = st.m1 = -INFINITY;
  st.l0 = st.l1 = 0.f;
}

// Fold keys [krow0, krow0 + kvalid) of buffer B (bias indices from 0) into the state.
__device__ __forceinline__ void state_attend(SoftmaxState& st, const AttnBuf& B, int krow0, int kvalid, float scale,
                                             int lane) {
  const int t4 = lane & 3;
  const int ntiles = (kvalid + 7) >> 3;
  const int kchunks = (kvalid + 15) >> 4;
#pragma unroll 1
  for (int sb = 0; sb * 64 < kvalid; ++sb) {
    const int nt_hi = ntiles - sb * 8;
    const int kc_hi = kchunks - sb * 4;
    const int kr = krow0 + sb * 64;
    float s[8][4];
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      if (nt < nt_hi) {
#pragma unroll
        for (int e = 0; e < 4; ++e) s[nt][e] = 0.f;
        uint32_t kb0, kb1, kb2, kb3;
        ldsm_x4(smem_u32(&B.k[kr + nt * 8 + (lane & 7)][(lane >> 3) * 8]), kb0, kb1, kb2, kb3);
        mma16816(s[nt], st.qa[0], kb0, kb1);
        mma16816(s[nt], st.qa[1], kb2, kb3);
        const float bias0 = B.bias[sb * 64 + nt * 8 + 2 * t4];
        const float bias1 = B.bias[sb * 64 + nt * 8 + 2 * t4 + 1];
        s[nt][0] = fmaf(s[nt][0], scale, bias0);
        s[nt][1] = fmaf(s[nt][1], scale, bias1);
        s[nt][2] = fmaf(s[nt][2], scale, bias0);
        s[nt][3] = fmaf(s[nt][3], scale, bias1);
        mx0 = fmaxf(mx0, fmaxf(s[nt][0], s[nt][1]));
        mx1 = fmaxf(mx1, fmaxf(s[nt][2], s[nt][3]));
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(st.m0, mx0), mn1 = fmaxf(st.m1, mx1);
    const float ref0 = mn0 == -INFINITY ? 0.f : mn0;
    const float ref1 = mn1 == -INFINITY ? 0.f : mn1;
    const float c0 = exp2f(st.m0 - ref0), c1 = exp2f(st.m1 - ref1);
    st.m0 = mn0;
    st.m1 = mn1;
    float ls0 = 0.f, ls1 = 0.f;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      if (nt < nt_hi) {
        s[nt][0] = exp2f(s[nt][0] - ref0);
        s[nt][1] = exp2f(s[nt][1] - ref0);
        s[nt][2] = exp2f(s[nt][2] - ref1);
        s[nt][3] = exp2f(s[nt][3] - ref1);
        ls0 += s[nt][0] + s[nt][1];
        ls1 += s[nt][2] + s[nt][3];
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) s[nt][e] = 0.f;
      }
    }
    st.l0 = st.l0 * c0 + ls0;
    st.l1 = st.l1 * c1 + ls1;
#pragma unroll
    for (int nd = 0; nd < 4; ++nd) {
      st.o[nd][0] *= c0;
      st.o[nd][1] *= c0;
      st.o[nd][2] *= c1;
      st.o[nd][3] *= c1;
    }
#pragma unroll
    for (int kc = 0; kc < 4; ++kc) {
      if (kc < kc_hi) {
        uint32_t pa[4];
        pa[0] = pack_half2(s[2 * kc][0], s[2 * kc][1]);
        pa[1] = pack_half2(s[2 * kc][2], s[2 * kc][3]);
        pa[2] = pack_half2(s[2 * kc + 1][0], s[2 * kc + 1][1]);
        pa[3] = pack_half2(s[2 * kc + 1][2], s[2 * kc + 1][3]);
#pragma unroll
        for (int dp = 0; dp < 2; ++dp) {
          const int mi = lane >> 3;
          const int r = kr + kc * 16 + (lane & 7) + (mi & 1) * 8;
          const int c = dp * 16 + (mi >> 1) * 8;
          uint32_t v0, v1, v2, v3;
          ldsm_x4_t(smem_u32(&B.v[r][c]), v0, v1, v2, v3);
          mma16816(st.o[dp * 2 + 0], pa, v0, v1);
          mma16816(st.o[dp * 2 + 1], pa, v2, v3);
        }
      }
    }
  }
}

// Normalise and store the 16 query rows starting at sentence row qr0 for head h.
__device__ __forceinline__ void state_store(const SoftmaxState& st, const AttnParams& p, int start, int len, int qr0,
                                            int h, int lane) {
  const int g = lane >> 2, t4 = lane & 3;
  float L0 = st.l0 + __shfl_xor_sync(0xffffffffu, st.l0, 1);
  L0 += __shfl_xor_sync(0xffffffffu, L0, 2);
  float L1 = st.l1 + __shfl_xor_sync(0xffffffffu, st.l1, 1);
  L1 += __shfl_xor_sync(0xffffffffu, L1, 2);
  const float inv0 = L0 > 0.f ? 1.0f / L0 : 0.f;
  const float inv1 = L1 > 0.f ? 1.0f / L1 : 0.f;
  const int r0 = qr0 + g;
  const int r1 = r0 + 8;
  const int col = h * kHeadDim + 2 * t4;
  __half* out0 = p.ctx + static_cast<size_t>(start + r0) * kHidden + col;
  __half* out1 = p.ctx + static_cast<size_t>(start + r1) * kHidden + col;
#pragma unroll
  for (int nd = 0; nd < 4; ++nd) {
    if (r0 < len) *reinterpret_cast<uint32_t*>(out0 + nd * 8) = pack_half2(st.o[nd][0] * inv0, st.o[nd][1] * inv0);
    if (r1 < len) *reinterpret_cast<uint32_t*>(out1 + nd * 8) = pack_half2(st.o[nd][2] * inv1, st.o[nd][3] * inv1);
  }
}

__global__ void __launch_bounds__(kAttnThreads, 3) attention_varlen_kernel(AttnParams p) {
  extern __shared__ __align__(16) uint8_t attn_smem[];
  AttnBuf* bufs = reinterpret_cast<AttnBuf*>(attn_smem);
  int* s_cu = reinterpret_cast<int*>(bufs + 2);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  const int batch = p.meta ? p.meta[0] : p.batch;
  const int max_len = p.meta ? p.meta[2] : p.max_len;
  // The key mask only exists for padded calls (meta[3] = 1); packed calls skip it.
  const uint8_t* tokmask = (p.meta && p.meta[3] == 0) ? nullptr : p.tokmask;
  Decomp d;
  d.qshift = 0;
  if (max_len > kKeyBlock)
    while ((kQRows << d.qshift) < max_len) ++d.qshift;
  d.items = (batch * kHeads) << d.qshift;
  const int* cu = p.cu;
  if (batch < kCuCache) {
    for (int i = tid; i <= batch; i += kAttnThreads) s_cu[i] = p.cu[i];
    __syncthreads();
    cu = s_cu;
  }

  Unit cur = find_unit(cu, d, blockIdx.x, gridDim.x, p.min_len);
  if (cur.item < 0) return;
  load_unit(p, tokmask, d, cur, bufs[0], tid);
  cp_async_commit();
  int bi = 0;
  Unit nxt = next_unit(cu, d, cur, gridDim.x, p.min_len);
  SoftmaxState st;

  while (cur.item >= 0) {
    if (nxt.item >= 0) {
      load_unit(p, tokmask, d, nxt, bufs[bi ^ 1], tid);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const AttnBuf& B = bufs[bi];
    const int hpc = heads_per_cta(cur.len);
    const int h0 = d.h(cur.item);
    if (cur.len > kKeyBlock) {
      // streamed: this warp's 16 rows of the 64-row chunk, key block kb
      const int qr0 = d.qc(cur.item) * kQRows + warp * 16;
      if (qr0 < cur.len) {
        if (cur.kb == 0) state_begin(st, B, warp * 16, lane);
        int kvalid = cur.len - cur.kb * kKeyBlock;
        kvalid = kvalid > kKeyBlock ? kKeyBlock : kvalid;
        state_attend(st, B, 0, kvalid, p.scale_log2, lane);
        if ((cur.kb + 1) * kKeyBlock >= cur.len) state_store(st, p, cur.start, cur.len, qr0, h0, lane);
      }
    } else {
      // whole sentence in the buffer: walk the query blocks of this warp's head slot
      const int wph = 4 / hpc;  // warps per head slot
      const int slot = warp / wph;
      const int kslot = kKeyBlock / hpc;
      const int qslot = hpc == 1 ? kKeyBlock : kQRows / hpc;
      for (int qb = warp % wph; qb * 16 < cur.len; qb += wph) {
        state_begin(st, B, slot * qslot + qb * 16, lane);
        state_attend(st, B, slot * kslot, cur.len, p.scale_log2, lane);
        state_store(st, p, cur.start, cur.len, qb * 16, h0 + slot, lane);
      }
    }
    const Unit nxt2 = next_unit(cu, d, nxt, gridDim.x, p.min_len);
    __syncthreads();  // buffer bi is refilled on the next iteration
    cur = nxt;
    nxt = nxt2;
    bi ^= 1;
  }
}

int attention_grid(int num_sms) { return num_sms * 3; }

cudaError_t launch_attention(const AttnParams& p, int grid, cudaStream_t stream) {
  constexpr int smem = 2 * static_cast<int>(sizeof(AttnBuf)) + kCuCache * 4;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attention_varlen_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  attention_varlen_kernel<<<grid, kAttnThreads, smem, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace bbh
