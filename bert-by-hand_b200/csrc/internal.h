// Internal launch interfaces shared between the kernel translation units and the C ABI.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <string>

struct bbh_ws;

namespace bbh {

// L2 access-policy window given to every launch of this thread while set (the forward's
// launches when the workspace keeps its weights persisting in L2), or null.
const cudaAccessPolicyWindow* current_l2_window();
void set_current_l2_window(const cudaAccessPolicyWindow* w);

// Launch with optional programmatic dependent launch (pdl) and cluster dimension.
template <typename... KArgs, typename... Args>
cudaError_t launch_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
                      int cluster, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[3];
  int na = 0;
  if (const cudaAccessPolicyWindow* apw = current_l2_window()) {
    attr[na].id = cudaLaunchAttributeAccessPolicyWindow;
    attr[na].val.accessPolicyWindow = *apw;
    ++na;
  }
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (cluster > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = static_cast<unsigned>(cluster);
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = static_cast<unsigned>(na);
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// ------------------------------------------------------------------ C ABI internals
// Sets the calling thread's bbh_last_error() message and returns code.
int internal_fail(int code, const std::string& msg);
// Device and capacity of a workspace.
void ws_limits(const bbh_ws* ws, int* device, int* max_tokens, int* max_batch, int* max_len);
// The workspace's slot for the corpus driver's staging state; free_fn releases it when
// the workspace is freed.
void** ws_corpus_stage(bbh_ws* ws, void (*free_fn)(void*));
// Number of compute lanes the corpus driver uses for this workspace (1 or 2).
int ws_corpus_lanes(const bbh_ws* ws);
// Gives dst (the corpus driver's second lane) src's launch settings: programmatic dependent
// launch, graph use, GEMM tiles and the L2 window.
void ws_inherit_settings(bbh_ws* dst, const bbh_ws* src);

// ------------------------------------------------------------------ GEMM (tcgen05)
enum Epilogue : int {
  kEpiBias = 0,      // C = A W^T + bias
  kEpiGelu = 1,      // C = gelu_erf(A W^T + bias)
  kEpiResLN = 2,     // C = LayerNorm(A W^T + bias + residual) * gamma + beta   (N == 384)
};

struct GemmParams {
  __half* C;
  int ldc;
  int N;
  int K;
  const __half* bias;      // [N] or null
  const __half* residual;  // [rows, ldr] (kEpiResLN)
  int ldr;
  const __half* gamma;     // [N] (kEpiResLN)
  const __half* beta;      // [N] (kEpiResLN)
  float eps;
  const int* rows_dev;     // when non-null the row count is read from device memory
  int rows;                // otherwise this host value is used
  int* err;                // device error word
};

struct GemmPlan {
  CUtensorMap tmA;
  CUtensorMap tmB;
  CUtensorMap tmC;
  CUtensorMap tmR;  // residual (kEpiResLN), set by set_gemm_residual
  CUtensorMap tmB2;  // W with (bn2 / 2)-row boxes for the CTA-pair kernel
  GemmParams p;
  int bn;
  int bn2;  // pair-tile width (CTA-pair kernel, gemm_pair.cu) or 0 for the one-SM kernel
  int epi;
  int grid;
  int rows_cap;
};

// Builds the tensor maps and picks the tile shape. A: [rows_cap, K] row-major with row
// stride lda elements; W: [N, K] row-major (nn.Linear layout); C: [rows_cap, N] with row
// stride ldc (written by TMA stores, clipped at rows_cap and N). Returns 0 or a BBH_ERR_*.
// pair_mode: 0 = one SM per 128-row tile; 1 = CTA pairs of 256 x 192 tiles where N allows
// it, else 256 x 256; 2 = 256 x 256 first.
int make_gemm_plan(GemmPlan* plan, const __half* A, int lda, int rows_cap, const __half* W, int N, int K,
                   __half* C, int ldc, int epi, int num_sms, int pair_mode);
// Tensor map of a row-major [rows, cols] fp16 matrix (row stride ld elements), box
// box_cols x box_rows with the given swizzle. Returns 0 or a BBH_ERR_*.
int encode_2d(CUtensorMap* map, const __half* base, int rows, int cols, int ld, int box_cols, int box_rows,
              CUtensorMapSwizzle swz);
// kEpiResLN: the residual [rows_cap, N] with row stride ldr (read with TMA, 16-byte aligned).
int set_gemm_residual(GemmPlan* plan, const __half* R, int ldr);
cudaError_t launch_gemm(const GemmPlan& plan, cudaStream_t stream, bool pdl = false);
// CTA-pair kernel (gemm_pair.cu): bias / GELU epilogues, N a multiple of the pair width.
bool gemm_pair_supported(int N, int epi, int bn);
cudaError_t launch_gemm_pair(const GemmPlan& plan, cudaStream_t stream, bool pdl);
// CTA-pair residual-LayerNorm GEMM over whole 384-wide rows (gemm_ln.cu).
cudaError_t launch_gemm_ln_pair(const GemmPlan& plan, cudaStream_t stream, bool pdl);
// Process-wide default tile mode (make_gemm_plan's pair_mode) for the unit operators and
// for workspaces created afterwards; a workspace keeps its own copy.
int default_gemm_pair_mode();
void set_default_gemm_pair_mode(int mode);

// ------------------------------------------------------------------ other kernels
// Forward-call description consumed by the first kernel of a forward. It is passed by
// value, so a captured graph can be re-pointed at new inputs by updating one node.
struct EmbedParams {
  const int32_t* ids;         // [T]
  const int32_t* types;       // [T] or null (all type 0)
  const int32_t* cu_seqlens;  // [B+1] device, packed mode; null in padded mode
  const int32_t* mask;        // [B*S] padded mode (null: all real)
  int batch;
  int seq;                    // padded mode row length (0 in packed mode)
  int total;                  // T
  int max_len;
  // model
  const __half* word;
  const __half* pos;
  const __half* type;
  const __half* gamma;
  const __half* beta;
  float eps;
  // outputs
  __half* out;                // [T, 384]
  int32_t* ws_cu;             // [B+1] copy of the segment offsets
  uint8_t* ws_tokmask;        // [T] 1 = real token (attends and is pooled)
  int32_t* ws_meta;           // {B, T, max_len, has_mask}
  int* err;
  int32_t* index_dump;        // [T, 4] or null: (word id, position, type id, mask) per token
};
cudaError_t launch_embed_ln(const EmbedParams& p, int grid, cudaStream_t stream, bool pdl = false);

struct AttnParams {
  const __half* qkv;       // [T, 1152]: Q | K | V, head h at columns h*32
  __half* ctx;             // [T, 384]
  const int32_t* cu;       // [B+1]
  const uint8_t* tokmask;  // [T], null = every key usable
  const int32_t* meta;     // {B, T, max_len, has_mask}, or null to use the host values below
  int batch;
  int max_len;
  int min_len;             // sentences shorter than this are skipped (the short-sentence kernel has them)
  float scale_log2;        // log2(e) / sqrt(head_dim)
};
// tcgen05 flash-style kernel for sentences of kAttnTcMaxLen+1 .. 512 tokens (min_len)
cudaError_t launch_attention_long(const AttnParams& p, int grid, cudaStream_t stream, bool pdl = false);
// tcgen05 kernel: sentences of at most kAttnTcMaxLen tokens
constexpr int kAttnTcMaxLen = 128;
cudaError_t launch_attention_tc(const AttnParams& p, int grid, cudaStream_t stream, bool pdl = false);

struct PoolParams {
  const __half* hidden;    // [T, 384]
  const int32_t* cu;       // [B+1]
  const uint8_t* tokmask;  // [T], null = every token pooled
  const int32_t* meta;     // {B, ...}, or null to use `batch`
  int batch;
  __half* emb;             // [B, 384]
};
const void* embed_kernel_fn();
const void* pool_kernel_fn();
cudaError_t launch_pool_l2(const PoolParams& p, int grid, cudaStream_t stream, bool pdl = false);

cudaError_t launch_layernorm(const __half* x, const __half* residual, const __half* gamma, const __half* beta,
                             __half* y, int rows, float eps, cudaStream_t stream);

}  // namespace bbh
