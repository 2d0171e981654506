// Example caller of the C++ drop-in API (include/bert_by_hand.hpp), written the way the
// reference's own callers are (tests/test_batch.cu:29-58, bench/bench.cu:31-49):
// load weights, make a workspace, copy ids/types/mask to the device, bert_embed, copy back.
//
//   bert_embed_main <weights_dir> <ids.bin> <types.bin> <mask.bin> <batch> <seq> <out.bin>
// ids/types/mask: int32 [batch*seq]; out: fp16 [batch*384].
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "bert_by_hand.hpp"

static std::vector<int32_t> read_i32(const char* path, size_t n) {
  std::vector<int32_t> v(n);
  FILE* f = std::fopen(path, "rb");
  if (!f || std::fread(v.data(), 4, n, f) != n) {
    std::fprintf(stderr, "cannot read %s\n", path);
    std::exit(2);
  }
  std::fclose(f);
  return v;
}

int main(int argc, char** argv) {
  if (argc != 8) {
    std::fprintf(stderr, "usage: %s weights ids types mask batch seq out\n", argv[0]);
    return 2;
  }
  const int batch = std::atoi(argv[5]), seq = std::atoi(argv[6]);
  const size_t n = size_t(batch) * seq;
  auto ids = read_i32(argv[2], n), types = read_i32(argv[3], n), mask = read_i32(argv[4], n);

  ModelWeights w = load_model_weights(argv[1]);
  Workspace ws = make_workspace(batch, seq);
  int32_t *d_ids, *d_types, *d_mask;
  __half* d_emb;
  cudaMalloc(&d_ids, n * 4);
  cudaMalloc(&d_types, n * 4);
  cudaMalloc(&d_mask, n * 4);
  cudaMalloc(&d_emb, size_t(batch) * model::HIDDEN * 2);
  cudaMemcpy(d_ids, ids.data(), n * 4, cudaMemcpyHostToDevice);
  cudaMemcpy(d_types, types.data(), n * 4, cudaMemcpyHostToDevice);
  cudaMemcpy(d_mask, mask.data(), n * 4, cudaMemcpyHostToDevice);

  bert_embed(ws, w, d_ids, d_types, d_mask, d_emb, batch, seq);
  bert_embed(ws, w, d_ids, d_types, d_mask, d_emb, batch, seq);  // graph replay path

  std::vector<__half> emb(size_t(batch) * model::HIDDEN);
  if (cudaMemcpy(emb.data(), d_emb, emb.size() * 2, cudaMemcpyDeviceToHost) != cudaSuccess) return 3;
  FILE* f = std::fopen(argv[7], "wb");
  std::fwrite(emb.data(), 2, emb.size(), f);
  std::fclose(f);
  cudaFree(d_ids);
  cudaFree(d_types);
  cudaFree(d_mask);
  cudaFree(d_emb);
  std::printf("bert_embed ok: batch %d seq %d\n", batch, seq);
  return 0;
}
