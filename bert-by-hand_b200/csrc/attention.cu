// Variable-length (cu_seqlens-packed) multi-head self-attention with online softmax.
// Replaces the reference's three-kernel attention (scores -> masked softmax -> context:
// src/kernels/attention.cu:17-121, src/kernels/softmax.cu:26-73, wired at
// src/model/encoder.cu:37-45), with no S x S buffer and no padding.
//
// Q, K and V are read as strided slices of the fused QKV buffer [T, 1152] (head h at
// columns h*32, 384 + h*32, 768 + h*32), and the context is written straight into the
// merged-heads layout [T, 384], as the reference does.
//
// Work item = (sentence, head, 64-query chunk); a 4-warp CTA owns one item, each warp
// 16 query rows. Keys are streamed in 64-key tiles through shared memory; scores and
// P.V use mma.sync m16n8k16 (fp16 in, fp32 accumulate), softmax runs in fp32 in the
// exp2 domain with a running max and sum per row. A key is dropped when it lies past the
// sentence end or its mask entry is 0 (src/kernels/softmax.cu:43-59). A row whose keys
// are all masked produces zeros, as the reference's softmax does.
#include "common.cuh"
#include "internal.h"

namespace bbh {

constexpr int kAttnThreads = 128;
constexpr int kTile = 64;
constexpr int kRowPad = 40;  // fp16 per smem row: 80 B keeps ldmatrix rows conflict-free

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

__global__ void __launch_bounds__(kAttnThreads) attention_varlen_kernel(AttnParams p) {
  __shared__ __align__(16) __half sQ[kTile][kRowPad];
  __shared__ __align__(16) __half sK[kTile][kRowPad];
  __shared__ __align__(16) __half sV[kTile][kRowPad];
  __shared__ float sBias[kTile];  // 0 for a usable key, -inf for a dropped one

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int g = lane >> 2;  // fragment row group
  const int t4 = lane & 3;  // fragment column pair

  const int batch = p.meta ? p.meta[0] : p.batch;
  const int max_len = p.meta ? p.meta[2] : p.max_len;
  const int qchunks = (max_len + kTile - 1) / kTile;
  const int items = batch * kHeads * qchunks;

  for (int item = blockIdx.x; item < items; item += gridDim.x) {
    const int qc = item % qchunks;
    const int h = (item / qchunks) % kHeads;
    const int b = item / (qchunks * kHeads);
    const int start = p.cu[b];
    const int len = p.cu[b + 1] - start;
    const int q0 = qc * kTile;
    if (q0 >= len) continue;  // uniform over the CTA

    const __half* base = p.qkv + static_cast<size_t>(start) * kQkvLd + h * kHeadDim;

    // Q tile: 64 rows x 32 fp16 = 256 16-byte pieces
    for (int i = tid; i < kTile * 4; i += kAttnThreads) {
      const int r = i >> 2, c = (i & 3) * 8;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (q0 + r < len) v = __ldg(reinterpret_cast<const uint4*>(base + static_cast<size_t>(q0 + r) * kQkvLd + c));
      *reinterpret_cast<uint4*>(&sQ[r][c]) = v;
    }
    __syncthreads();

    const bool active = q0 + warp * 16 < len;
    uint32_t qa[2][4];
    if (active) {
#pragma unroll
      for (int kc = 0; kc < 2; ++kc) {
        const int mi = lane >> 3;
        const int r = warp * 16 + (lane & 7) + (mi & 1) * 8;
        const int c = kc * 16 + (mi >> 1) * 8;
        ldsm_x4(smem_u32(&sQ[r][c]), qa[kc][0], qa[kc][1], qa[kc][2], qa[kc][3]);
      }
    }

    float o[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) o[i][j] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

    for (int k0 = 0; k0 < len; k0 += kTile) {
      for (int i = tid; i < kTile * 4; i += kAttnThreads) {
        const int r = i >> 2, c = (i & 3) * 8;
        uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
        if (k0 + r < len) {
          const __half* rowp = base + static_cast<size_t>(k0 + r) * kQkvLd + c;
          kv = __ldg(reinterpret_cast<const uint4*>(rowp + kHidden));
          vv = __ldg(reinterpret_cast<const uint4*>(rowp + 2 * kHidden));
        }
        *reinterpret_cast<uint4*>(&sK[r][c]) = kv;
        *reinterpret_cast<uint4*>(&sV[r][c]) = vv;
      }
      if (tid < kTile) {
        const int j = k0 + tid;
        sBias[tid] = (j < len && (!p.tokmask || p.tokmask[start + j])) ? 0.f : -INFINITY;
      }
      __syncthreads();

      if (active) {
        float s[8][4];
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
          for (int e = 0; e < 4; ++e) s[nt][e] = 0.f;
          uint32_t kb0, kb1, kb2, kb3;
          ldsm_x4(smem_u32(&sK[nt * 8 + (lane & 7)][(lane >> 3) * 8]), kb0, kb1, kb2, kb3);
          mma16816(s[nt], qa[0], kb0, kb1);
          mma16816(s[nt], qa[1], kb2, kb3);
        }
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
          const float bias0 = sBias[nt * 8 + 2 * t4];
          const float bias1 = sBias[nt * 8 + 2 * t4 + 1];
          s[nt][0] = s[nt][0] * p.scale_log2 + bias0;
          s[nt][1] = s[nt][1] * p.scale_log2 + bias1;
          s[nt][2] = s[nt][2] * p.scale_log2 + bias0;
          s[nt][3] = s[nt][3] * p.scale_log2 + bias1;
          mx0 = fmaxf(mx0, fmaxf(s[nt][0], s[nt][1]));
          mx1 = fmaxf(mx1, fmaxf(s[nt][2], s[nt][3]));
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
        const float ref0 = mn0 == -INFINITY ? 0.f : mn0;
        const float ref1 = mn1 == -INFINITY ? 0.f : mn1;
        const float c0 = exp2f(m0 - ref0), c1 = exp2f(m1 - ref1);
        m0 = mn0;
        m1 = mn1;
        float ls0 = 0.f, ls1 = 0.f;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
          s[nt][0] = exp2f(s[nt][0] - ref0);
          s[nt][1] = exp2f(s[nt][1] - ref0);
          s[nt][2] = exp2f(s[nt][2] - ref1);
          s[nt][3] = exp2f(s[nt][3] - ref1);
          ls0 += s[nt][0] + s[nt][1];
          ls1 += s[nt][2] + s[nt][3];
        }
        l0 = l0 * c0 + ls0;
        l1 = l1 * c1 + ls1;
#pragma unroll
        for (int nd = 0; nd < 4; ++nd) {
          o[nd][0] *= c0;
          o[nd][1] *= c0;
          o[nd][2] *= c1;
          o[nd][3] *= c1;
        }
#pragma unroll
        for (int kc = 0; kc < 4; ++kc) {
          uint32_t pa[4];
          pa[0] = pack_half2(s[2 * kc][0], s[2 * kc][1]);
          pa[1] = pack_half2(s[2 * kc][2], s[2 * kc][3]);
          pa[2] = pack_half2(s[2 * kc + 1][0], s[2 * kc + 1][1]);
          pa[3] = pack_half2(s[2 * kc + 1][2], s[2 * kc + 1][3]);
#pragma unroll
          for (int dp = 0; dp < 2; ++dp) {
            const int mi = lane >> 3;
            const int r = kc * 16 + (lane & 7) + (mi & 1) * 8;
            const int c = dp * 16 + (mi >> 1) * 8;
            uint32_t v0, v1, v2, v3;
            ldsm_x4_t(smem_u32(&sV[r][c]), v0, v1, v2, v3);
            mma16816(o[dp * 2 + 0], pa, v0, v1);
            mma16816(o[dp * 2 + 1], pa, v2, v3);
          }
        }
      }
      __syncthreads();
    }

    if (active) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
      l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
      l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
      l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
      const float inv0 = l0 > 0.f ? 1.0f / l0 : 0.f;
      const float inv1 = l1 > 0.f ? 1.0f / l1 : 0.f;
      const int r0 = q0 + warp * 16 + g;
      const int r1 = r0 + 8;
      __half* out0 = p.ctx + static_cast<size_t>(start + r0) * kHidden + h * kHeadDim + 2 * t4;
      __half* out1 = p.ctx + static_cast<size_t>(start + r1) * kHidden + h * kHeadDim + 2 * t4;
#pragma unroll
      for (int nd = 0; nd < 4; ++nd) {
        if (r0 < len) *reinterpret_cast<uint32_t*>(out0 + nd * 8) = pack_half2(o[nd][0] * inv0, o[nd][1] * inv0);
        if (r1 < len) *reinterpret_cast<uint32_t*>(out1 + nd * 8) = pack_half2(o[nd][2] * inv1, o[nd][3] * inv1);
      }
    }
  }
}

int attention_grid(int num_sms) { return num_sms * 8; }

cudaError_t launch_attention(const AttnParams& p, int grid, cudaStream_t stream) {
  attention_varlen_kernel<<<grid, kAttnThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace bbh
