// Test-only C entry points over the REFERENCE's own CUDA implementation, compiled from the
// unmodified sources under the reference tree (see oracle/Makefile). Used by the GPU
// parity tests as a second oracle and to time the reference's kernels on a B200.
//
// The reference reads weights from "weights/<HF key>.bin" relative to the working
// directory (src/core/model_config.h:19, src/core/loader.h:10-16), so each call switches
// into the directory that holds "weights/".
#include <unistd.h>

#include <cstdint>
#include <cstring>
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

}  // extern "C"
