// Test-only C entry points over the REFERENCE's own CUDA implementation, compiled from the
// unmodified sources under the reference tree (see oracle/Makefile). Used by the GPU
// parity tests as a second oracle and to time the reference's kernels on a B200.
//
// The reference reads weights from "weights/<HF key>.bin" relative to the working
// directory (src/core/model_config.h:19, src/core/loader.h:10-16), so each call switches
// into the directory that holds "weights/".
#include <unistd.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <numeric>
#include <string>
#include <vector>

#include "core/device_buffer.h"
#include "model/forward.h"
#include "model/weights.h"
#include "model/workspace.h"

namespace {
struct Cwd {
  char old[4096];
  explicit Cwd(const char* dir) {
    if (!getcwd(old, sizeof(old))) old[0] = 0;
    if (chdir(dir) != 0) old[0] = 0;
  }
  ~Cwd() {
    if (old[0] && chdir(old) != 0) old[0] = 0;
  }
};
}  // namespace

extern "C" {

// emb_host: [batch, 384] fp16 bits. seq must be <= 128 and a multiple of 16 (reference
// preconditions, src/model/workspace.h:20-36, src/kernels/attention.cu:100-110).
int ref_embed(const char* root, const int32_t* ids, const int32_t* types, const int32_t* mask, uint16_t* emb_host,
              int batch, int seq, int iters, float* ms_per_forward) {
  if (seq > model::SEQ_LEN || seq % 16) return -1;
  Cwd cd(root);
  ModelWeights w = load_model_weights();
  Workspace ws = make_workspace(batch);
  const size_t n = size_t(batch) * seq;
  DeviceBuffer di(n * 4), dt(n * 4), dm(n * 4), de(size_t(batch) * model::HIDDEN * 2);
  di.from_host(ids, n * 4);
  dt.from_host(types, n * 4);
  dm.from_host(mask, n * 4);
  auto* ep = static_cast<__half*>(de.data());
  bert_embed(ws, w, static_cast<const int32_t*>(di.data()), static_cast<const int32_t*>(dt.data()),
             static_cast<const int32_t*>(dm.data()), ep, batch, seq);
  if (iters > 0 && ms_per_forward) {
    for (int i = 0; i < 3; ++i)
      bert_embed(ws, w, static_cast<const int32_t*>(di.data()), static_cast<const int32_t*>(dt.data()),
                 static_cast<const int32_t*>(dm.data()), ep, batch, seq);
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    cudaEventRecord(a);
    for (int i = 0; i < iters; ++i)
      bert_embed(ws, w, static_cast<const int32_t*>(di.data()), static_cast<const int32_t*>(dt.data()),
                 static_cast<const int32_t*>(dm.data()), ep, batch, seq);
    cudaEventRecord(b);
    cudaEventSynchronize(b);
    float ms = 0;
    cudaEventElapsedTime(&ms, a, b);
    *ms_per_forward = ms / iters;
    cudaEventDestroy(a);
    cudaEventDestroy(b);
  }
  de.to_host(emb_host, size_t(batch) * model::HIDDEN * 2);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

// The reference's dynamic-length corpus loop (bench/corpus.cu:80-128): sentences sorted by
// length, cut into batches of B, each padded to its longest sentence rounded up to 16 (at
// least 16), all batches resident on the device, one bert_embed per batch. Sentences come
// packed (ids [cu[n]], cu [n+1]); each must be <= 128 tokens (the reference's SEQ_LEN).
// Times `iters` passes over the corpus with CUDA events after one untimed pass and writes
// ms per pass; emb_host (optional, [n, 384] fp16 bits) receives the embeddings in corpus
// order.
int ref_corpus(const char* root, const int32_t* ids, const int32_t* cu, int n, int B, int iters,
               float* ms_per_pass, uint16_t* emb_host) {
  if (n <= 0 || B <= 0) return -1;
  for (int i = 0; i < n; ++i)
    if (cu[i + 1] - cu[i] < 1 || cu[i + 1] - cu[i] > model::SEQ_LEN) return -1;
  Cwd cd(root);
  ModelWeights w = load_model_weights();
  Workspace ws = make_workspace(B);
  std::vector<int> order(n);
  std::iota(order.begin(), order.end(), 0);
  std::stable_sort(order.begin(), order.end(),
                   [&](int a, int b) { return cu[a + 1] - cu[a] < cu[b + 1] - cu[b]; });
  struct Batch {
    DeviceBuffer ids, types, mask;
    int size, eff, start;
  };
  std::vector<Batch> batches;
  for (int s = 0; s < n; s += B) {
    const int bs = std::min(B, n - s);
    int mx = 0;
    for (int k = 0; k < bs; ++k) mx = std::max(mx, cu[order[s + k] + 1] - cu[order[s + k]]);
    const int eff = std::max(16, (mx + 15) / 16 * 16);
    std::vector<int32_t> hi(size_t(bs) * eff, 0), ht(size_t(bs) * eff, 0), hm(size_t(bs) * eff, 0);
    for (int k = 0; k < bs; ++k) {
      const int si = order[s + k], L = cu[si + 1] - cu[si];
      for (int j = 0; j < L; ++j) {
        hi[size_t(k) * eff + j] = ids[cu[si] + j];
        hm[size_t(k) * eff + j] = 1;
      }
    }
    Batch b{DeviceBuffer(hi.size() * 4), DeviceBuffer(ht.size() * 4), DeviceBuffer(hm.size() * 4), bs, eff, s};
    b.ids.from_host(hi.data(), hi.size() * 4);
    b.types.from_host(ht.data(), ht.size() * 4);
    b.mask.from_host(hm.data(), hm.size() * 4);
    batches.push_back(std::move(b));
  }
  DeviceBuffer de(size_t(n) * model::HIDDEN * 2);
  auto* ep = static_cast<__half*>(de.data());
  auto pass = [&]() {
    for (auto& b : batches)
      bert_embed(ws, w, static_cast<const int32_t*>(b.ids.data()), static_cast<const int32_t*>(b.types.data()),
                 static_cast<const int32_t*>(b.mask.data()), ep + size_t(b.start) * model::HIDDEN, b.size, b.eff);
  };
  pass();
  if (iters > 0 && ms_per_pass) {
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    cudaEventRecord(a);
    for (int i = 0; i < iters; ++i) pass();
    cudaEventRecord(b);
    cudaEventSynchronize(b);
    float ms = 0;
    cudaEventElapsedTime(&ms, a, b);
    *ms_per_pass = ms / iters;
    cudaEventDestroy(a);
    cudaEventDestroy(b);
  }
  if (emb_host) {
    std::vector<uint16_t> h(size_t(n) * model::HIDDEN);
    de.to_host(h.data(), h.size() * 2);
    for (int i = 0; i < n; ++i)
      std::memcpy(emb_host + size_t(order[i]) * model::HIDDEN, h.data() + size_t(i) * model::HIDDEN,
                  model::HIDDEN * 2);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

}  // extern "C"
