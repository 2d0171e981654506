// C ABI: weights arena, workspace, forward orchestration (one CUDA graph per workspace)
// and the unit operators. Mirrors the reference's host API (src/model/forward.cu,
// weights.h, workspace.h) with status codes instead of abort().
#include "common.cuh"
#include "internal.h"
#include "../../include/bbh.h"

#include <cmath>
#include <cstdio>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

using bbh::GemmPlan;

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(BBH_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

#define BBH_CUDA(call)                                  \
  do {                                                  \
    cudaError_t e_ = (call);                            \
    if (e_ != cudaSuccess) return cuda_fail(e_, #call); \
  } while (0)

// ------------------------------------------------------------------ tensor catalogue
struct Spec {
  std::string name;
  int64_t numel;
};

std::vector<Spec> specs_for(int layers) {
  using namespace bbh;
  std::vector<Spec> s = {
      {"embeddings.word_embeddings.weight", int64_t(kVocab) * kHidden},
      {"embeddings.position_embeddings.weight", int64_t(kMaxPos) * kHidden},
      {"embeddings.token_type_embeddings.weight", int64_t(kTypes) * kHidden},
      {"embeddings.LayerNorm.weight", kHidden},
      {"embeddings.LayerNorm.bias", kHidden},
  };
  for (int i = 0; i < layers; ++i) {
    const std::string p = "encoder.layer." + std::to_string(i) + ".";
    for (const char* part : {"query", "key", "value"}) {
      s.push_back({p + "attention.self." + part + ".weight", int64_t(kHidden) * kHidden});
      s.push_back({p + "attention.self." + part + ".bias", kHidden});
    }
    s.push_back({p + "attention.output.dense.weight", int64_t(kHidden) * kHidden});
    s.push_back({p + "attention.output.dense.bias", kHidden});
    s.push_back({p + "attention.output.LayerNorm.weight", kHidden});
    s.push_back({p + "attention.output.LayerNorm.bias", kHidden});
    s.push_back({p + "intermediate.dense.weight", int64_t(kFfn) * kHidden});
    s.push_back({p + "intermediate.dense.bias", kFfn});
    s.push_back({p + "output.dense.weight", int64_t(kHidden) * kFfn});
    s.push_back({p + "output.dense.bias", kHidden});
    s.push_back({p + "output.LayerNorm.weight", kHidden});
    s.push_back({p + "output.LayerNorm.bias", kHidden});
  }
  return s;
}

const std::vector<Spec>& cached_specs(int layers) {
  static std::mutex mu;
  static std::vector<Spec> s6, s12;
  std::lock_guard<std::mutex> lk(mu);
  std::vector<Spec>& s = layers == 12 ? s12 : s6;
  if (s.empty()) s = specs_for(layers);
  return s;
}

bool valid_layers(int layers) { return layers == 6 || layers == 12; }

int g_num_sms(int device) {
  static int cache[64] = {};
  if (device >= 0 && device < 64 && cache[device] > 0) return cache[device];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0) n = 148;
  if (device >= 0 && device < 64) cache[device] = n;
  return n;
}

// Per-device error word for the unit operators (which run without a workspace).
int* unit_err_word(int device) {
  static std::mutex mu;
  static int* words[64] = {};
  std::lock_guard<std::mutex> lk(mu);
  if (device < 0 || device >= 64) return nullptr;
  if (!words[device]) {
    int* p = nullptr;
    if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) return nullptr;
    cudaMemset(p, 0, sizeof(int));
    words[device] = p;
  }
  return words[device];
}

int check_sm100(int device) {
  static std::mutex mu;
  static signed char ok[64] = {};  // 0 unknown, 1 sm_100, -1 other
  if (device < 0 || device >= 64) return fail(BBH_ERR_ARG, "bad device ordinal");
  {
    std::lock_guard<std::mutex> lk(mu);
    if (ok[device] == 1) return BBH_OK;
  }
  int major = 0;
  cudaError_t e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
  std::lock_guard<std::mutex> lk(mu);
  ok[device] = major == 10 ? 1 : -1;
  if (major != 10) return fail(BBH_ERR_UNSUPPORTED, "libbbh needs an sm_100 (B200-class) GPU");
  return BBH_OK;
}

}  // namespace

// ====================================================================== weights

struct LayerPtrs {
  const __half *qkv_w, *qkv_b, *o_w, *o_b, *ln1_g, *ln1_b, *i_w, *i_b, *o2_w, *o2_b, *ln2_g, *ln2_b;
};

struct bbh_weights {
  int device = 0;
  int layers = 6;
  __half* arena = nullptr;
  size_t arena_elems = 0;
  const __half *word, *pos, *type, *emb_g, *emb_b;
  std::vector<LayerPtrs> L;
};

static size_t align128(size_t n) { return (n + 127) & ~size_t(127); }

extern "C" {

const char* bbh_last_error(void) { return g_last_error.c_str(); }

int bbh_num_tensors(int layers) { return valid_layers(layers) ? 5 + 16 * layers : 0; }

const char* bbh_tensor_name(int layers, int index) {
  if (!valid_layers(layers) || index < 0 || index >= bbh_num_tensors(layers)) return nullptr;
  return cached_specs(layers)[index].name.c_str();
}

int64_t bbh_tensor_numel(int layers, int index) {
  if (!valid_layers(layers) || index < 0 || index >= bbh_num_tensors(layers)) return -1;
  return cached_specs(layers)[index].numel;
}

int bbh_weights_from_host(const uint16_t* const* tensors, int layers, int device, bbh_weights** out) {
  using namespace bbh;
  if (!tensors || !out || !valid_layers(layers)) return fail(BBH_ERR_ARG, "bbh_weights_from_host: bad arguments");
  *out = nullptr;
  const auto& specs = cached_specs(layers);
  for (size_t i = 0; i < specs.size(); ++i)
    if (!tensors[i]) return fail(BBH_ERR_ARG, "bbh_weights_from_host: null tensor " + specs[i].name);
  int rc = check_sm100(device);
  if (rc) return rc;
  BBH_CUDA(cudaSetDevice(device));

  // Arena order: embeddings, then per layer qkv_w qkv_b o_w o_b ln1 i_w i_b o2_w o2_b ln2,
  // each piece 256-byte aligned. Q, K and V stack along the output dimension.
  std::vector<size_t> off;
  size_t total = 0;
  auto take = [&](size_t n) {
    off.push_back(total);
    total += align128(n);
  };
  take(size_t(kVocab) * kHidden);
  take(size_t(kMaxPos) * kHidden);
  take(size_t(kTypes) * kHidden);
  take(kHidden);
  take(kHidden);
  for (int l = 0; l < layers; ++l) {
    take(size_t(kQkvLd) * kHidden);
    take(kQkvLd);
    take(size_t(kHidden) * kHidden);
    take(kHidden);
    take(kHidden);
    take(kHidden);
    take(size_t(kFfn) * kHidden);
    take(kFfn);
    take(size_t(kHidden) * kFfn);
    take(kHidden);
    take(kHidden);
    take(kHidden);
  }
  std::vector<uint16_t> host(total, 0);
  auto put = [&](size_t dst, int idx) {
    std::memcpy(host.data() + dst, tensors[idx], size_t(specs[idx].numel) * 2);
  };
  for (int i = 0; i < 5; ++i) put(off[i], i);
  for (int l = 0; l < layers; ++l) {
    const int t = 5 + 16 * l;   // tensor index base (q.w q.b k.w k.b v.w v.b o.w o.b ln ln i.w i.b o2.w o2.b ln ln)
    const int o = 5 + 12 * l;   // arena piece base
    for (int j = 0; j < 3; ++j) {
      put(off[o + 0] + size_t(j) * kHidden * kHidden, t + 2 * j);
      put(off[o + 1] + size_t(j) * kHidden, t + 2 * j + 1);
    }
    for (int j = 0; j < 10; ++j) put(off[o + 2 + j], t + 6 + j);
  }

  bbh_weights* w = new bbh_weights();
  w->device = device;
  w->layers = layers;
  w->arena_elems = total;
  cudaError_t e = cudaMalloc(&w->arena, total * 2);
  if (e != cudaSuccess) {
    delete w;
    return cuda_fail(e, "cudaMalloc(weights)");
  }
  e = cudaMemcpy(w->arena, host.data(), total * 2, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(w->arena);
    delete w;
    return cuda_fail(e, "cudaMemcpy(weights)");
  }
  const __half* a = w->arena;
  w->word = a + off[0];
  w->pos = a + off[1];
  w->type = a + off[2];
  w->emb_g = a + off[3];
  w->emb_b = a + off[4];
  for (int l = 0; l < layers; ++l) {
    const int o = 5 + 12 * l;
    LayerPtrs lp;
    const __half** f = &lp.qkv_w;
    for (int j = 0; j < 12; ++j) f[j] = a + off[o + j];
    w->L.push_back(lp);
  }
  *out = w;
  return BBH_OK;
}

int bbh_weights_load(const char* dir, int layers, int device, bbh_weights** out) {
  if (!dir || !out || !valid_layers(layers)) return fail(BBH_ERR_ARG, "bbh_weights_load: bad arguments");
  const auto& specs = cached_specs(layers);
  std::vector<std::vector<uint16_t>> data(specs.size());
  std::vector<const uint16_t*> ptrs(specs.size());
  for (size_t i = 0; i < specs.size(); ++i) {
    const std::string path = std::string(dir) + "/" + specs[i].name + ".bin";
    FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) return fail(BBH_ERR_IO, "cannot open " + path);
    data[i].resize(size_t(specs[i].numel));
    const size_t got = std::fread(data[i].data(), 2, data[i].size(), f);
    std::fclose(f);
    if (got != data[i].size())
      return fail(BBH_ERR_IO, path + ": expected " + std::to_string(data[i].size()) + " elements, got " +
                                  std::to_string(got));
    ptrs[i] = data[i].data();
  }
  return bbh_weights_from_host(ptrs.data(), layers, device, out);
}

void bbh_weights_free(bbh_weights* w) {
  if (!w) return;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(w->device);
  cudaFree(w->arena);
  cudaSetDevice(prev);
  delete w;
}

int bbh_weights_layers(const bbh_weights* w) { return w ? w->layers : 0; }

}  // extern "C"

// ====================================================================== workspace

struct bbh_ws {
  int device = 0;
  int num_sms = 148;
  const bbh_weights* w = nullptr;
  int max_tokens = 0, max_batch = 0, max_len = 0;
  void* arena = nullptr;
  __half *X = nullptr, *Y = nullptr, *qkv = nullptr, *ctx = nullptr, *inter = nullptr;
  uint8_t* tokmask = nullptr;
  int32_t* cu = nullptr;
  int32_t* meta = nullptr;
  int* err = nullptr;
  std::vector<GemmPlan> plans;  // 4 per layer: QKV, O+LN, FFN1+GELU, FFN2+LN
  int gemm_pairs = 2;           // make_gemm_plan's pair_mode for this workspace's plans
  bool plans_stale = false;     // the plans must be rebuilt (tile mode changed)
  bool l2_persist = false;      // forward launches carry an L2 access-policy window over the layer weights
  cudaAccessPolicyWindow l2_window{};
  bool pdl = true;                      // programmatic dependent launch between the forward's kernels
  bool use_graph = true;
  cudaStream_t cap_stream = nullptr;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  cudaGraphNode_t n_embed = nullptr, n_pool = nullptr;
  cudaKernelNodeParams kp_embed{}, kp_pool{};
  bbh::EmbedParams ep{};
  bbh::PoolParams pp{};
  // per-kernel timing
  bool timing = false;
  std::vector<cudaEvent_t> ev;  // pairs
  std::vector<int> ev_kind;
  size_t ev_used = 0;
  // host corpus driver staging (csrc/corpus.cu), created on first use
  void* corpus_stage = nullptr;
  void (*corpus_stage_free)(void*) = nullptr;
  int corpus_lanes = 1;
};

namespace {
void drop_graph(bbh_ws* ws);
}

namespace bbh {
namespace {
thread_local const cudaAccessPolicyWindow* t_l2_window = nullptr;
}
const cudaAccessPolicyWindow* current_l2_window() { return t_l2_window; }
void set_current_l2_window(const cudaAccessPolicyWindow* w) { t_l2_window = w; }
int internal_fail(int code, const std::string& msg) { return fail(code, msg); }
void ws_limits(const bbh_ws* ws, int* device, int* max_tokens, int* max_batch, int* max_len) {
  *device = ws->device;
  *max_tokens = ws->max_tokens;
  *max_batch = ws->max_batch;
  *max_len = ws->max_len;
}
void** ws_corpus_stage(bbh_ws* ws, void (*free_fn)(void*)) {
  ws->corpus_stage_free = free_fn;
  return &ws->corpus_stage;
}
int ws_corpus_lanes(const bbh_ws* ws) { return ws->corpus_lanes; }
void ws_inherit_settings(bbh_ws* dst, const bbh_ws* src) {
  if (dst->pdl != src->pdl || dst->use_graph != src->use_graph || dst->gemm_pairs != src->gemm_pairs ||
      dst->l2_persist != src->l2_persist || std::memcmp(&dst->l2_window, &src->l2_window, sizeof(dst->l2_window))) {
    drop_graph(dst);
    if (dst->gemm_pairs != src->gemm_pairs) dst->plans_stale = true;  // rebuilt with src's tiles
    dst->pdl = src->pdl;
    dst->use_graph = src->use_graph;
    dst->gemm_pairs = src->gemm_pairs;
    dst->l2_persist = src->l2_persist;
    dst->l2_window = src->l2_window;
  }
}
}  // namespace bbh

namespace {

int build_plans(bbh_ws* ws, const bbh_weights* w) {
  using namespace bbh;
  ws->plans.assign(size_t(w->layers) * 4, GemmPlan{});
  const int pm = ws->gemm_pairs;
  for (int l = 0; l < w->layers; ++l) {
    const LayerPtrs& L = w->L[l];
    GemmPlan* P = &ws->plans[size_t(l) * 4];
    const int T = ws->max_tokens;
    int rc = make_gemm_plan(&P[0], ws->X, kHidden, T, L.qkv_w, kQkvLd, kHidden, ws->qkv, kQkvLd, kEpiBias,
                            ws->num_sms, pm);
    if (!rc)
      rc = make_gemm_plan(&P[1], ws->ctx, kHidden, T, L.o_w, kHidden, kHidden, ws->Y, kHidden, kEpiResLN, ws->num_sms,
                          pm);
    if (!rc)
      rc = make_gemm_plan(&P[2], ws->Y, kHidden, T, L.i_w, kFfn, kHidden, ws->inter, kFfn, kEpiGelu, ws->num_sms, pm);
    if (!rc)
      rc = make_gemm_plan(&P[3], ws->inter, kFfn, T, L.o2_w, kHidden, kFfn, ws->X, kHidden, kEpiResLN, ws->num_sms,
                          pm);
    if (!rc) rc = set_gemm_residual(&P[1], ws->X, kHidden);
    if (!rc) rc = set_gemm_residual(&P[3], ws->Y, kHidden);
    if (rc) return fail(rc, "tensor map encoding failed");
    P[0].p.C = ws->qkv;  P[0].p.ldc = kQkvLd; P[0].p.bias = L.qkv_b;
    P[1].p.C = ws->Y;    P[1].p.ldc = kHidden; P[1].p.bias = L.o_b;
    P[1].p.gamma = L.ln1_g; P[1].p.beta = L.ln1_b;
    P[2].p.C = ws->inter; P[2].p.ldc = kFfn; P[2].p.bias = L.i_b;
    P[3].p.C = ws->X;    P[3].p.ldc = kHidden; P[3].p.bias = L.o2_b;
    P[3].p.gamma = L.ln2_g; P[3].p.beta = L.ln2_b;
    for (int j = 0; j < 4; ++j) {
      P[j].p.rows_dev = ws->meta + 1;
      P[j].p.err = ws->err;
      P[j].p.eps = 1e-12f;
    }
  }
  ws->w = w;
  return BBH_OK;
}

void drop_graph(bbh_ws* ws) {
  if (ws->exec) cudaGraphExecDestroy(ws->exec);
  if (ws->graph) cudaGraphDestroy(ws->graph);
  ws->exec = nullptr;
  ws->graph = nullptr;
  ws->n_embed = ws->n_pool = nullptr;
}

// Event pair around one launch when per-kernel timing is on.
struct KernelMark {
  bbh_ws* ws;
  cudaStream_t s;
  size_t slot = SIZE_MAX;
  KernelMark(bbh_ws* w, cudaStream_t st, int kind) : ws(w), s(st) {
    if (!ws->timing) return;
    if (ws->ev_used + 2 > ws->ev.size()) {
      for (int i = 0; i < 64; ++i) {
        cudaEvent_t e;
        if (cudaEventCreate(&e) != cudaSuccess) return;
        ws->ev.push_back(e);
      }
      ws->ev_kind.resize(ws->ev.size() / 2);
    }
    slot = ws->ev_used;
    ws->ev_used += 2;
    ws->ev_kind[slot / 2] = kind;
    cudaEventRecord(ws->ev[slot], s);
  }
  ~KernelMark() {
    if (slot != SIZE_MAX) cudaEventRecord(ws->ev[slot + 1], s);
  }
};

// Enqueue one forward. pool == false stops after the last layer (encode). dump, when
// non-null, receives (layers+1) snapshots of the hidden state (eager mode only).
int enqueue_forward_launches(bbh_ws* ws, const bbh::EmbedParams& ep, bool pool, const bbh::PoolParams& pp,
                             __half* dump, int total, cudaStream_t s);

// The forward's launches, with the workspace's L2 window (if any) on each of them.
int enqueue_forward(bbh_ws* ws, const bbh::EmbedParams& ep, bool pool, const bbh::PoolParams& pp, __half* dump,
                    int total, cudaStream_t s) {
  struct WindowScope {
    explicit WindowScope(const cudaAccessPolicyWindow* w) { bbh::set_current_l2_window(w); }
    ~WindowScope() { bbh::set_current_l2_window(nullptr); }
  } scope(ws->l2_persist ? &ws->l2_window : nullptr);
  return enqueue_forward_launches(ws, ep, pool, pp, dump, total, s);
}

int enqueue_forward_launches(bbh_ws* ws, const bbh::EmbedParams& ep, bool pool, const bbh::PoolParams& pp,
                             __half* dump, int total, cudaStream_t s) {
  using namespace bbh;
  const int L = ws->w->layers;
  const int row_grid = ws->num_sms * 8;
  {
    KernelMark km(ws, s, 0);
    BBH_CUDA(launch_embed_ln(ep, row_grid, s, ws->pdl));
  }
  const size_t plane = size_t(total) * kHidden;
  if (dump) BBH_CUDA(cudaMemcpyAsync(dump, ws->X, plane * 2, cudaMemcpyDeviceToDevice, s));
  AttnParams ap{};
  ap.qkv = ws->qkv;
  ap.ctx = ws->ctx;
  ap.cu = ws->cu;
  ap.tokmask = ws->tokmask;
  ap.meta = ws->meta;
  ap.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(double(kHeadDim)));
  for (int l = 0; l < L; ++l) {
    const GemmPlan* P = &ws->plans[size_t(l) * 4];
    {
      KernelMark km(ws, s, 1);
      BBH_CUDA(launch_gemm(P[0], s, ws->pdl));
    }
    {
      KernelMark km(ws, s, 2);
      ap.min_len = 0;
      BBH_CUDA(launch_attention_tc(ap, 4 * ws->num_sms, s, ws->pdl));
      if (ws->max_len > kAttnTcMaxLen) {
        ap.min_len = kAttnTcMaxLen + 1;
        BBH_CUDA(launch_attention_long(ap, 2 * ws->num_sms, s, ws->pdl));
      }
    }
    {
      KernelMark km(ws, s, 3);
      BBH_CUDA(launch_gemm(P[1], s, ws->pdl));
    }
    for (int j = 2; j < 4; ++j) {
      KernelMark km(ws, s, 2 + j);
      BBH_CUDA(launch_gemm(P[j], s, ws->pdl));
    }
    if (dump) BBH_CUDA(cudaMemcpyAsync(dump + plane * (l + 1), ws->X, plane * 2, cudaMemcpyDeviceToDevice, s));
  }
  if (pool) {
    int grid = ws->max_batch < ws->num_sms * 16 ? ws->max_batch : ws->num_sms * 16;
    KernelMark km(ws, s, 6);
    BBH_CUDA(launch_pool_l2(pp, grid, s, ws->pdl));
  }
  return BBH_OK;
}

int capture_graph(bbh_ws* ws, const bbh::EmbedParams& ep, const bbh::PoolParams& pp) {
  drop_graph(ws);
  if (!ws->cap_stream) BBH_CUDA(cudaStreamCreateWithFlags(&ws->cap_stream, cudaStreamNonBlocking));
  BBH_CUDA(cudaStreamBeginCapture(ws->cap_stream, cudaStreamCaptureModeThreadLocal));
  int rc = enqueue_forward(ws, ep, true, pp, nullptr, ep.total, ws->cap_stream);
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamEndCapture(ws->cap_stream, &g);
  if (rc) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture");
  ws->graph = g;
  size_t n = 0;
  BBH_CUDA(cudaGraphGetNodes(g, nullptr, &n));
  std::vector<cudaGraphNode_t> nodes(n);
  BBH_CUDA(cudaGraphGetNodes(g, nodes.data(), &n));
  for (auto nd : nodes) {
    cudaGraphNodeType ty;
    BBH_CUDA(cudaGraphNodeGetType(nd, &ty));
    if (ty != cudaGraphNodeTypeKernel) continue;
    cudaKernelNodeParams kp;
    BBH_CUDA(cudaGraphKernelNodeGetParams(nd, &kp));
    if (kp.func == bbh::embed_kernel_fn()) {
      ws->n_embed = nd;
      ws->kp_embed = kp;
    } else if (kp.func == bbh::pool_kernel_fn()) {
      ws->n_pool = nd;
      ws->kp_pool = kp;
    }
  }
  if (!ws->n_embed || !ws->n_pool) return fail(BBH_ERR_CUDA, "graph capture lost the embed/pool nodes");
  BBH_CUDA(cudaGraphInstantiate(&ws->exec, g, 0));
  return BBH_OK;
}

int run_embed(bbh_ws* ws, const bbh::EmbedParams& ep, const bbh::PoolParams& pp, cudaStream_t s) {
  if (!ws->use_graph || ws->timing) return enqueue_forward(ws, ep, true, pp, nullptr, ep.total, s);
  if (!ws->exec) {
    int rc = capture_graph(ws, ep, pp);
    if (rc) {
      drop_graph(ws);
      return rc;
    }
  } else {
    ws->ep = ep;
    ws->pp = pp;
    void* a1[1] = {&ws->ep};
    void* a2[1] = {&ws->pp};
    cudaKernelNodeParams k1 = ws->kp_embed, k2 = ws->kp_pool;
    k1.kernelParams = a1;
    k1.extra = nullptr;
    k2.kernelParams = a2;
    k2.extra = nullptr;
    BBH_CUDA(cudaGraphExecKernelNodeSetParams(ws->exec, ws->n_embed, &k1));
    BBH_CUDA(cudaGraphExecKernelNodeSetParams(ws->exec, ws->n_pool, &k2));
  }
  BBH_CUDA(cudaGraphLaunch(ws->exec, s));
  return BBH_OK;
}

int prepare(bbh_ws* ws, const bbh_weights* w) {
  if (!ws || !w) return fail(BBH_ERR_ARG, "null workspace or weights");
  if (w->device != ws->device) return fail(BBH_ERR_ARG, "weights and workspace are on different devices");
  BBH_CUDA(cudaSetDevice(ws->device));
  if (ws->w != w || ws->plans_stale) {
    drop_graph(ws);
    int rc = build_plans(ws, w);
    if (rc) return rc;
    ws->plans_stale = false;
  }
  return BBH_OK;
}

bbh::EmbedParams base_embed_params(bbh_ws* ws, const bbh_weights* w) {
  bbh::EmbedParams ep{};
  ep.word = w->word;
  ep.pos = w->pos;
  ep.type = w->type;
  ep.gamma = w->emb_g;
  ep.beta = w->emb_b;
  ep.eps = 1e-12f;
  ep.out = ws->X;
  ep.ws_cu = ws->cu;
  ep.ws_tokmask = ws->tokmask;
  ep.ws_meta = ws->meta;
  ep.err = ws->err;
  return ep;
}

bbh::PoolParams base_pool_params(bbh_ws* ws, uint16_t* emb) {
  bbh::PoolParams pp{};
  pp.hidden = ws->X;
  pp.cu = ws->cu;
  pp.tokmask = ws->tokmask;
  pp.meta = ws->meta;
  pp.emb = reinterpret_cast<__half*>(emb);
  return pp;
}

bool misaligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) != 0; }

int check_padded(bbh_ws* ws, const int32_t* ids, const void* out, int batch, int seq) {
  if (!ids || !out) return fail(BBH_ERR_ARG, "null ids or output pointer");
  if (misaligned16(out)) return fail(BBH_ERR_ARG, "the output must be 16-byte aligned");
  if (batch <= 0 || seq <= 0) return fail(BBH_ERR_ARG, "batch and seq must be positive");
  if (seq > BBH_MAX_POSITIONS) return fail(BBH_ERR_ARG, "seq exceeds the 512-entry position table");
  if (batch > ws->max_batch || seq > ws->max_len || int64_t(batch) * seq > ws->max_tokens)
    return fail(BBH_ERR_CAPACITY, "batch x seq exceeds the workspace capacity");
  return BBH_OK;
}

int check_packed(bbh_ws* ws, const int32_t* ids, const int32_t* cu, const void* out, int batch, int total,
                 int max_len) {
  if (!ids || !cu || !out) return fail(BBH_ERR_ARG, "null ids, cu_seqlens or output pointer");
  if (misaligned16(out)) return fail(BBH_ERR_ARG, "the output must be 16-byte aligned");
  if (batch <= 0 || total < 0 || max_len <= 0) return fail(BBH_ERR_ARG, "bad batch / total_tokens / max_len");
  if (max_len > BBH_MAX_POSITIONS) return fail(BBH_ERR_ARG, "max_len exceeds the 512-entry position table");
  if (batch > ws->max_batch || total > ws->max_tokens || max_len > ws->max_len)
    return fail(BBH_ERR_CAPACITY, "request exceeds the workspace capacity");
  return BBH_OK;
}

}  // namespace

extern "C" {

int bbh_ws_create(const bbh_weights* w, int max_tokens, int max_batch, int max_len, bbh_ws** out) {
  using namespace bbh;
  if (!w || !out || max_tokens <= 0 || max_batch <= 0 || max_len <= 0 || max_len > BBH_MAX_POSITIONS)
    return fail(BBH_ERR_ARG, "bbh_ws_create: bad arguments");
  *out = nullptr;
  BBH_CUDA(cudaSetDevice(w->device));
  bbh_ws* ws = new bbh_ws();
  ws->device = w->device;
  ws->num_sms = g_num_sms(w->device);
  ws->max_tokens = max_tokens;
  ws->max_batch = max_batch;
  ws->max_len = max_len;
  ws->gemm_pairs = bbh::default_gemm_pair_mode();
  const size_t T = size_t(max_tokens);
  size_t sizes[9] = {T * kHidden * 2, T * kHidden * 2, T * kQkvLd * 2, T * kHidden * 2, T * kFfn * 2,
                     T, size_t(max_batch + 1) * 4, 16, 16};
  size_t total = 0, offs[9];
  for (int i = 0; i < 9; ++i) {
    offs[i] = total;
    total += (sizes[i] + 255) & ~size_t(255);
  }
  cudaError_t e = cudaMalloc(&ws->arena, total);
  if (e != cudaSuccess) {
    delete ws;
    return cuda_fail(e, "cudaMalloc(workspace)");
  }
  cudaMemset(ws->arena, 0, total);
  uint8_t* b = static_cast<uint8_t*>(ws->arena);
  ws->X = reinterpret_cast<__half*>(b + offs[0]);
  ws->Y = reinterpret_cast<__half*>(b + offs[1]);
  ws->qkv = reinterpret_cast<__half*>(b + offs[2]);
  ws->ctx = reinterpret_cast<__half*>(b + offs[3]);
  ws->inter = reinterpret_cast<__half*>(b + offs[4]);
  ws->tokmask = b + offs[5];
  ws->cu = reinterpret_cast<int32_t*>(b + offs[6]);
  ws->meta = reinterpret_cast<int32_t*>(b + offs[7]);
  ws->err = reinterpret_cast<int*>(b + offs[8]);
  int rc = build_plans(ws, w);
  if (rc) {
    bbh_ws_free(ws);
    return rc;
  }
  *out = ws;
  return BBH_OK;
}

void bbh_ws_free(bbh_ws* ws) {
  if (!ws) return;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(ws->device);
  if (ws->corpus_stage && ws->corpus_stage_free) ws->corpus_stage_free(ws->corpus_stage);
  drop_graph(ws);
  if (ws->cap_stream) cudaStreamDestroy(ws->cap_stream);
  for (auto e : ws->ev) cudaEventDestroy(e);
  cudaFree(ws->arena);
  cudaSetDevice(prev);
  delete ws;
}

int bbh_ws_set_pdl(bbh_ws* ws, int enable) {
  if (!ws) return fail(BBH_ERR_ARG, "null workspace");
  if ((enable != 0) != ws->pdl) {
    ws->pdl = enable != 0;
    drop_graph(ws);
  }
  return BBH_OK;
}

int bbh_ws_set_corpus_lanes(bbh_ws* ws, int lanes) {
  if (!ws || lanes < 1 || lanes > 2) return fail(BBH_ERR_ARG, "bbh_ws_set_corpus_lanes: lanes must be 1 or 2");
  ws->corpus_lanes = lanes;
  return BBH_OK;
}

int bbh_set_gemm_pairs(int mode) {
  if (mode < 0 || mode > 2) return fail(BBH_ERR_ARG, "bbh_set_gemm_pairs: mode must be 0, 1 or 2");
  bbh::set_default_gemm_pair_mode(mode);
  return BBH_OK;
}

int bbh_ws_set_gemm_pairs(bbh_ws* ws, int mode) {
  if (!ws) return fail(BBH_ERR_ARG, "null workspace");
  if (mode < 0 || mode > 2) return fail(BBH_ERR_ARG, "bbh_ws_set_gemm_pairs: mode must be 0, 1 or 2");
  if (mode != ws->gemm_pairs) {
    ws->gemm_pairs = mode;
    drop_graph(ws);
    ws->plans_stale = true;  // the plans are rebuilt with the new tiles by the next forward
  }
  return BBH_OK;
}

int bbh_ws_set_l2_persist(bbh_ws* ws, int enable) {
  if (!ws) return fail(BBH_ERR_ARG, "null workspace");
  if (!enable) {
    if (ws->l2_persist) drop_graph(ws);
    ws->l2_persist = false;
    return BBH_OK;
  }
  if (!ws->w) return fail(BBH_ERR_ARG, "bbh_ws_set_l2_persist: the workspace has no weights yet");
  BBH_CUDA(cudaSetDevice(ws->device));
  int max_persist = 0, max_window = 0;
  BBH_CUDA(cudaDeviceGetAttribute(&max_persist, cudaDevAttrMaxPersistingL2CacheSize, ws->device));
  BBH_CUDA(cudaDeviceGetAttribute(&max_window, cudaDevAttrMaxAccessPolicyWindowSize, ws->device));
  if (max_persist <= 0 || max_window <= 0) return fail(BBH_ERR_UNSUPPORTED, "no persisting L2 on this device");
  // the encoder layers' weights: from the first layer's QKV weight to the end of the arena
  const bbh_weights* w = ws->w;
  const __half* lo = w->L.front().qkv_w;
  size_t bytes = size_t(w->arena + w->arena_elems - lo) * sizeof(__half);
  if (bytes > size_t(max_window)) bytes = size_t(max_window);
  size_t limit = 0;
  BBH_CUDA(cudaDeviceGetLimit(&limit, cudaLimitPersistingL2CacheSize));
  const size_t want = bytes < size_t(max_persist) ? bytes : size_t(max_persist);
  // context-scoped: the set-aside ends with this process's CUDA context
  if (limit < want) BBH_CUDA(cudaDeviceSetLimit(cudaLimitPersistingL2CacheSize, want));
  ws->l2_window.base_ptr = const_cast<__half*>(lo);
  ws->l2_window.num_bytes = bytes;
  ws->l2_window.hitRatio = static_cast<float>(double(want) / double(bytes));
  ws->l2_window.hitProp = cudaAccessPropertyPersisting;
  ws->l2_window.missProp = cudaAccessPropertyStreaming;
  ws->l2_persist = true;
  drop_graph(ws);
  return BBH_OK;
}

int bbh_ws_set_graph(bbh_ws* ws, int enable) {
  if (!ws) return fail(BBH_ERR_ARG, "null workspace");
  ws->use_graph = enable != 0;
  if (!ws->use_graph) drop_graph(ws);
  return BBH_OK;
}

int bbh_device_error(bbh_ws* ws, int reset) {
  if (!ws) return fail(BBH_ERR_ARG, "null workspace");
  BBH_CUDA(cudaSetDevice(ws->device));
  BBH_CUDA(cudaDeviceSynchronize());
  int v = 0;
  BBH_CUDA(cudaMemcpy(&v, ws->err, sizeof(int), cudaMemcpyDeviceToHost));
  if (reset && v) BBH_CUDA(cudaMemset(ws->err, 0, sizeof(int)));
  return v;
}

int bbh_ws_set_kernel_timing(bbh_ws* ws, int enable) {
  if (!ws) return fail(BBH_ERR_ARG, "null workspace");
  ws->timing = enable != 0;
  return BBH_OK;
}

int bbh_ws_kernel_times(bbh_ws* ws, double* ms, int64_t* counts) {
  if (!ws || !ms || !counts) return fail(BBH_ERR_ARG, "bbh_ws_kernel_times: bad arguments");
  BBH_CUDA(cudaSetDevice(ws->device));
  for (size_t i = 0; i + 1 < ws->ev_used; i += 2) {
    BBH_CUDA(cudaEventSynchronize(ws->ev[i + 1]));
    float t = 0.f;
    BBH_CUDA(cudaEventElapsedTime(&t, ws->ev[i], ws->ev[i + 1]));
    const int k = ws->ev_kind[i / 2];
    ms[k] += t;
    counts[k] += 1;
  }
  ws->ev_used = 0;
  return BBH_OK;
}

int bbh_launches_per_forward(const bbh_ws* ws) {
  if (!ws || !ws->w) return 0;
  const int per_layer = ws->max_len > bbh::kAttnTcMaxLen ? 6 : 5;
  return 2 + per_layer * ws->w->layers;
}

int bbh_embed(bbh_ws* ws, const bbh_weights* w, const int32_t* ids, const int32_t* types, const int32_t* mask,
              uint16_t* emb, int batch, int seq, void* stream) {
  int rc = prepare(ws, w);
  if (rc) return rc;
  rc = check_padded(ws, ids, emb, batch, seq);
  if (rc) return rc;
  bbh::EmbedParams ep = base_embed_params(ws, w);
  ep.ids = ids;
  ep.types = types;
  ep.mask = mask;
  ep.batch = batch;
  ep.seq = seq;
  ep.total = batch * seq;
  ep.max_len = seq;
  return run_embed(ws, ep, base_pool_params(ws, emb), static_cast<cudaStream_t>(stream));
}

int bbh_embed_varlen(bbh_ws* ws, const bbh_weights* w, const int32_t* ids, const int32_t* types,
                     const int32_t* cu_seqlens, int batch, int total_tokens, int max_len, uint16_t* emb,
                     void* stream) {
  int rc = prepare(ws, w);
  if (rc) return rc;
  rc = check_packed(ws, ids, cu_seqlens, emb, batch, total_tokens, max_len);
  if (rc) return rc;
  bbh::EmbedParams ep = base_embed_params(ws, w);
  ep.ids = ids;
  ep.types = types;
  ep.cu_seqlens = cu_seqlens;
  ep.batch = batch;
  ep.total = total_tokens;
  ep.max_len = max_len;
  return run_embed(ws, ep, base_pool_params(ws, emb), static_cast<cudaStream_t>(stream));
}

static int encode_common(bbh_ws* ws, const bbh::EmbedParams& ep, uint16_t* out, uint16_t* dump, cudaStream_t s) {
  bbh::PoolParams none{};
  int rc = enqueue_forward(ws, ep, false, none, reinterpret_cast<__half*>(dump), ep.total, s);
  if (rc) return rc;
  BBH_CUDA(cudaMemcpyAsync(out, ws->X, size_t(ep.total) * bbh::kHidden * 2, cudaMemcpyDeviceToDevice, s));
  return BBH_OK;
}

int bbh_encode(bbh_ws* ws, const bbh_weights* w, const int32_t* ids, const int32_t* types, const int32_t* mask,
               uint16_t* out, int batch, int seq, void* stream) {
  int rc = prepare(ws, w);
  if (rc) return rc;
  rc = check_padded(ws, ids, out, batch, seq);
  if (rc) return rc;
  bbh::EmbedParams ep = base_embed_params(ws, w);
  ep.ids = ids;
  ep.types = types;
  ep.mask = mask;
  ep.batch = batch;
  ep.seq = seq;
  ep.total = batch * seq;
  ep.max_len = seq;
  return encode_common(ws, ep, out, nullptr, static_cast<cudaStream_t>(stream));
}

int bbh_encode_varlen(bbh_ws* ws, const bbh_weights* w, const int32_t* ids, const int32_t* types,
                      const int32_t* cu_seqlens, int batch, int total_tokens, int max_len, uint16_t* out,
                      uint16_t* layer_dump, void* stream) {
  int rc = prepare(ws, w);
  if (rc) return rc;
  rc = check_packed(ws, ids, cu_seqlens, out, batch, total_tokens, max_len);
  if (rc) return rc;
  bbh::EmbedParams ep = base_embed_params(ws, w);
  ep.ids = ids;
  ep.types = types;
  ep.cu_seqlens = cu_seqlens;
  ep.batch = batch;
  ep.total = total_tokens;
  ep.max_len = max_len;
  return encode_common(ws, ep, out, layer_dump, static_cast<cudaStream_t>(stream));
}

int bbh_embed_gather_indices(bbh_ws* ws, const bbh_weights* w, const int32_t* ids, const int32_t* types,
                             const int32_t* mask, const int32_t* cu_seqlens, int batch, int seq, int total_tokens,
                             int max_len, int32_t* indices, void* stream) {
  int rc = prepare(ws, w);
  if (rc) return rc;
  if (!indices || (reinterpret_cast<uintptr_t>(indices) & 15))
    return fail(BBH_ERR_ARG, "bbh_embed_gather_indices: indices must be a 16-byte aligned [T, 4] int32 array");
  bbh::EmbedParams ep = base_embed_params(ws, w);
  ep.ids = ids;
  ep.types = types;
  ep.batch = batch;
  if (cu_seqlens) {
    rc = check_packed(ws, ids, cu_seqlens, indices, batch, total_tokens, max_len);
    if (rc) return rc;
    ep.cu_seqlens = cu_seqlens;
    ep.total = total_tokens;
    ep.max_len = max_len;
  } else {
    rc = check_padded(ws, ids, indices, batch, seq);
    if (rc) return rc;
    ep.mask = mask;
    ep.seq = seq;
    ep.total = batch * seq;
    ep.max_len = seq;
  }
  ep.index_dump = indices;
  BBH_CUDA(bbh::launch_embed_ln(ep, ws->num_sms * 8, static_cast<cudaStream_t>(stream)));
  return BBH_OK;
}

// ---------------------------------------------------------------------- unit operators

static int current_device(int* dev) {
  BBH_CUDA(cudaGetDevice(dev));
  return check_sm100(*dev);
}

static int unit_gemm(const uint16_t* A, const uint16_t* W, const uint16_t* bias, const uint16_t* residual,
                     const uint16_t* gamma, const uint16_t* beta, float eps, uint16_t* C, int M, int N, int K,
                     int epi, void* stream) {
  using namespace bbh;
  if (!A || !W || !C || M <= 0) return fail(BBH_ERR_ARG, "bbh_linear: bad arguments");
  if (epi == kEpiResLN && (!bias || !residual || !gamma || !beta))
    return fail(BBH_ERR_ARG, "residual LayerNorm needs bias, residual, gamma and beta");
  if ((reinterpret_cast<uintptr_t>(C) | reinterpret_cast<uintptr_t>(bias) |
       reinterpret_cast<uintptr_t>(residual)) & 15)
    return fail(BBH_ERR_ARG, "pointers must be 16-byte aligned");
  int dev = 0;
  int rc = current_device(&dev);
  if (rc) return rc;
  GemmPlan plan;
  rc = make_gemm_plan(&plan, reinterpret_cast<const __half*>(A), K, M, reinterpret_cast<const __half*>(W), N, K,
                      reinterpret_cast<__half*>(C), N, epi, g_num_sms(dev), default_gemm_pair_mode());
  if (rc) return fail(rc, "bbh_linear: unsupported shape or alignment (N, K must be multiples of 8)");
  plan.p.C = reinterpret_cast<__half*>(C);
  plan.p.ldc = N;
  plan.p.bias = reinterpret_cast<const __half*>(bias);
  if (epi == kEpiResLN) {
    rc = set_gemm_residual(&plan, reinterpret_cast<const __half*>(residual), N);
    if (rc) return fail(rc, "bbh_linear_residual_layernorm: residual tensor map encoding failed");
  }
  plan.p.gamma = reinterpret_cast<const __half*>(gamma);
  plan.p.beta = reinterpret_cast<const __half*>(beta);
  plan.p.eps = eps;
  plan.p.rows_dev = nullptr;
  plan.p.rows = M;
  plan.p.err = unit_err_word(dev);
  BBH_CUDA(launch_gemm(plan, static_cast<cudaStream_t>(stream)));
  return BBH_OK;
}

int bbh_linear(const uint16_t* A, const uint16_t* W, const uint16_t* bias, uint16_t* C, int M, int N, int K,
               int gelu, void* stream) {
  return unit_gemm(A, W, bias, nullptr, nullptr, nullptr, 0.f, C, M, N, K, gelu ? bbh::kEpiGelu : bbh::kEpiBias,
                   stream);
}

int bbh_linear_residual_layernorm(const uint16_t* A, const uint16_t* W, const uint16_t* bias,
                                  const uint16_t* residual, const uint16_t* gamma, const uint16_t* beta, float eps,
                                  uint16_t* C, int M, int K, void* stream) {
  return unit_gemm(A, W, bias, residual, gamma, beta, eps, C, M, bbh::kHidden, K, bbh::kEpiResLN, stream);
}

int bbh_layernorm(const uint16_t* x, const uint16_t* gamma, const uint16_t* beta, uint16_t* y, int M, int D,
                  float eps, const uint16_t* residual, void* stream) {
  if (!x || !gamma || !beta || !y || M < 0) return fail(BBH_ERR_ARG, "bbh_layernorm: bad arguments");
  if (D != bbh::kHidden) return fail(BBH_ERR_ARG, "bbh_layernorm: D must be 384");
  int dev = 0;
  int rc = current_device(&dev);
  if (rc) return rc;
  BBH_CUDA(bbh::launch_layernorm(reinterpret_cast<const __half*>(x), reinterpret_cast<const __half*>(residual),
                                 reinterpret_cast<const __half*>(gamma), reinterpret_cast<const __half*>(beta),
                                 reinterpret_cast<__half*>(y), M, eps, static_cast<cudaStream_t>(stream)));
  return BBH_OK;
}

int bbh_attention_varlen(const uint16_t* qkv, uint16_t* ctx, const int32_t* cu_seqlens, const uint8_t* keymask,
                         int batch, int max_len, void* stream) {
  if (!qkv || !ctx || !cu_seqlens || batch < 0 || max_len <= 0)
    return fail(BBH_ERR_ARG, "bbh_attention_varlen: bad arguments");
  int dev = 0;
  int rc = current_device(&dev);
  if (rc) return rc;
  bbh::AttnParams ap{};
  ap.qkv = reinterpret_cast<const __half*>(qkv);
  ap.ctx = reinterpret_cast<__half*>(ctx);
  ap.cu = cu_seqlens;
  ap.tokmask = keymask;
  ap.meta = nullptr;
  ap.batch = batch;
  ap.max_len = max_len;
  ap.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(double(bbh::kHeadDim)));
  BBH_CUDA(bbh::launch_attention_tc(ap, 4 * g_num_sms(dev), static_cast<cudaStream_t>(stream)));
  if (max_len > bbh::kAttnTcMaxLen) {
    ap.min_len = bbh::kAttnTcMaxLen + 1;
    BBH_CUDA(bbh::launch_attention_long(ap, 2 * g_num_sms(dev), static_cast<cudaStream_t>(stream)));
  }
  return BBH_OK;
}

int bbh_mean_pool_l2(const uint16_t* hidden, const int32_t* cu_seqlens, const uint8_t* tokmask, int batch,
                     uint16_t* emb, void* stream) {
  if (!hidden || !cu_seqlens || !emb || batch < 0) return fail(BBH_ERR_ARG, "bbh_mean_pool_l2: bad arguments");
  if (misaligned16(hidden) || misaligned16(emb))
    return fail(BBH_ERR_ARG, "bbh_mean_pool_l2: hidden and emb must be 16-byte aligned");
  int dev = 0;
  int rc = current_device(&dev);
  if (rc) return rc;
  bbh::PoolParams pp{};
  pp.hidden = reinterpret_cast<const __half*>(hidden);
  pp.cu = cu_seqlens;
  pp.tokmask = tokmask;
  pp.meta = nullptr;
  pp.batch = batch;
  pp.emb = reinterpret_cast<__half*>(emb);
  const int grid = batch < g_num_sms(dev) * 16 ? (batch > 0 ? batch : 1) : g_num_sms(dev) * 16;
  BBH_CUDA(bbh::launch_pool_l2(pp, grid, static_cast<cudaStream_t>(stream)));
  return BBH_OK;
}

}  // extern "C"

// ====================================================================== no-allocation path
// bbh_embed_varlen_static: the packed forward with all scratch in one file-scope device
// array (no cudaMalloc/cudaFree anywhere on this path). Host code must not pass the
// array's name to a kernel -- in host code it is only a stand-in for the symbol -- so the
// device address is looked up once per device with cudaGetSymbolAddress.

namespace {

constexpr size_t static_align(size_t n) { return (n + 255) & ~size_t(255); }
constexpr size_t kStT = BBH_STATIC_MAX_TOKENS;
constexpr size_t kStOffX = 0;
constexpr size_t kStOffY = kStOffX + static_align(kStT * bbh::kHidden * 2);
constexpr size_t kStOffQkv = kStOffY + static_align(kStT * bbh::kHidden * 2);
constexpr size_t kStOffCtx = kStOffQkv + static_align(kStT * bbh::kQkvLd * 2);
constexpr size_t kStOffInter = kStOffCtx + static_align(kStT * bbh::kHidden * 2);
constexpr size_t kStOffTok = kStOffInter + static_align(kStT * bbh::kFfn * 2);
constexpr size_t kStOffCu = kStOffTok + static_align(kStT);
constexpr size_t kStOffMeta = kStOffCu + static_align((BBH_STATIC_MAX_BATCH + 1) * 4);
constexpr size_t kStOffErr = kStOffMeta + static_align(16);
constexpr size_t kStBytes = kStOffErr + static_align(4);

}  // namespace

static __device__ __align__(256) unsigned char g_bbh_static_scratch[kStBytes];

namespace {

std::mutex g_static_mu;

// Device address of g_bbh_static_scratch on `device` (looked up with that device current).
int static_scratch(int device, uint8_t** out) {
  static uint8_t* addr[64] = {};
  if (device < 0 || device >= 64) return fail(BBH_ERR_ARG, "bad device ordinal");
  std::lock_guard<std::mutex> lk(g_static_mu);
  if (!addr[device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_bbh_static_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(static scratch)");
    addr[device] = static_cast<uint8_t*>(p);
  }
  *out = addr[device];
  return BBH_OK;
}

// GEMM plans (tensor maps over the static array and a weight arena) cached per device, so
// a call re-encodes them only when it is given a different weight arena. The arena's
// address and layer count determine every weight pointer, so they are the cache key.
struct StaticPlans {
  const __half* arena = nullptr;
  int layers = 0;
  std::vector<GemmPlan> plans;
};

int static_plans(bbh_ws* ws, const bbh_weights* w) {
  static StaticPlans cache[64];
  std::lock_guard<std::mutex> lk(g_static_mu);
  StaticPlans& c = cache[ws->device];
  if (c.arena != w->arena || c.layers != w->layers) {
    c.arena = nullptr;
    const int rc = build_plans(ws, w);
    if (rc) return rc;
    c.plans = ws->plans;
    c.arena = w->arena;
    c.layers = w->layers;
    return BBH_OK;
  }
  ws->plans = c.plans;
  ws->w = w;
  return BBH_OK;
}

}  // namespace

extern "C" {

int bbh_embed_varlen_static(const bbh_weights* w, const int32_t* ids, const int32_t* types,
                            const int32_t* cu_seqlens, int batch, int total_tokens, int max_len, uint16_t* emb,
                            void* stream) {
  if (!w || !ids || !cu_seqlens || !emb) return fail(BBH_ERR_ARG, "bbh_embed_varlen_static: null pointer");
  if (misaligned16(emb)) return fail(BBH_ERR_ARG, "bbh_embed_varlen_static: emb must be 16-byte aligned");
  if (batch <= 0 || total_tokens < 0 || max_len <= 0)
    return fail(BBH_ERR_ARG, "bbh_embed_varlen_static: bad batch / total_tokens / max_len");
  if (total_tokens > BBH_STATIC_MAX_TOKENS || batch > BBH_STATIC_MAX_BATCH || max_len > BBH_MAX_POSITIONS)
    return fail(BBH_ERR_CAPACITY, "bbh_embed_varlen_static: request exceeds the static scratch (at most " +
                                      std::to_string(BBH_STATIC_MAX_TOKENS) + " tokens, " +
                                      std::to_string(BBH_STATIC_MAX_BATCH) + " sentences, 512 per sentence)");
  BBH_CUDA(cudaSetDevice(w->device));
  uint8_t* base = nullptr;
  int rc = static_scratch(w->device, &base);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  // A workspace view of the static array (host-side bookkeeping only).
  bbh_ws ws;
  ws.device = w->device;
  ws.num_sms = g_num_sms(w->device);
  ws.max_tokens = BBH_STATIC_MAX_TOKENS;
  ws.max_batch = BBH_STATIC_MAX_BATCH;
  ws.max_len = max_len;  // the long-sentence attention kernel runs only when a sentence can need it
  ws.X = reinterpret_cast<__half*>(base + kStOffX);
  ws.Y = reinterpret_cast<__half*>(base + kStOffY);
  ws.qkv = reinterpret_cast<__half*>(base + kStOffQkv);
  ws.ctx = reinterpret_cast<__half*>(base + kStOffCtx);
  ws.inter = reinterpret_cast<__half*>(base + kStOffInter);
  ws.tokmask = base + kStOffTok;
  ws.cu = reinterpret_cast<int32_t*>(base + kStOffCu);
  ws.meta = reinterpret_cast<int32_t*>(base + kStOffMeta);
  ws.err = reinterpret_cast<int*>(base + kStOffErr);
  ws.use_graph = false;
  rc = static_plans(&ws, w);
  if (rc) return rc;

  // The error word must start at zero; everything else is written before it is read.
  BBH_CUDA(cudaMemsetAsync(ws.err, 0, sizeof(int), s));
  bbh::EmbedParams ep = base_embed_params(&ws, w);
  ep.ids = ids;
  ep.types = types;
  ep.cu_seqlens = cu_seqlens;
  ep.batch = batch;
  ep.total = total_tokens;
  ep.max_len = max_len;
  return enqueue_forward(&ws, ep, true, base_pool_params(&ws, emb), nullptr, total_tokens, s);
}

int bbh_static_device_error(void) {
  int dev = 0;
  BBH_CUDA(cudaGetDevice(&dev));
  uint8_t* base = nullptr;
  int rc = static_scratch(dev, &base);
  if (rc) return rc;
  BBH_CUDA(cudaDeviceSynchronize());
  int v = 0;
  BBH_CUDA(cudaMemcpy(&v, base + kStOffErr, sizeof(int), cudaMemcpyDeviceToHost));
  return v;
}

}  // extern "C"
