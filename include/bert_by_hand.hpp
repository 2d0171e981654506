// bert_by_hand.hpp -- C++ drop-in for tytrdev/bert-by-hand's host API, over libbbh.so.
//
// Same names, argument order and failure behaviour as the reference:
//   ModelWeights load_model_weights()                     src/model/weights.h:88-107
//   Workspace make_workspace(int batch = 1)               src/model/workspace.h:20-36
//   void bert_encode(ws, w, ids, types, mask, out, batch, seq)   src/model/forward.h:11-13
//   void bert_embed(ws, w, ids, types, mask, emb, batch, seq)    src/model/forward.h:17-19
// Pointers are device pointers; calls are asynchronous on the legacy default stream (or
// the stream given as the optional last argument). As in the reference
// (src/core/cuda_check.h:7-17) any failure prints a message and aborts. The engine
// underneath is the packed/graph-captured sm_100a implementation in libbbh.so.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <utility>
#include <vector>

#include "bbh.h"

namespace model {
constexpr int VOCAB_SIZE = 30522;
constexpr int HIDDEN = 384;
constexpr int NUM_LAYERS = 6;
constexpr int NUM_HEADS = 12;
constexpr int HEAD_DIM = 32;
constexpr int FFN_DIM = 1536;
constexpr int MAX_POSITION = 512;
constexpr int TYPE_VOCAB_SIZE = 2;
constexpr float LAYER_NORM_EPS = 1e-12f;
constexpr int SEQ_LEN = 128;
constexpr const char* WEIGHTS_DIR = "weights";
}  // namespace model

namespace bbh_detail {
inline void check(int rc, const char* what) {
  if (rc != BBH_OK) {
    std::fprintf(stderr, "%s failed (%d): %s\n", what, rc, bbh_last_error());
    std::abort();
  }
}
}  // namespace bbh_detail

// Device-resident weights (one arena). Move-only like the reference's DeviceBuffer members.
struct ModelWeights {
  bbh_weights* handle = nullptr;
  ModelWeights() = default;
  explicit ModelWeights(bbh_weights* h) : handle(h) {}
  ModelWeights(const ModelWeights&) = delete;
  ModelWeights& operator=(const ModelWeights&) = delete;
  ModelWeights(ModelWeights&& o) noexcept : handle(std::exchange(o.handle, nullptr)) {}
  ModelWeights& operator=(ModelWeights&& o) noexcept {
    if (this != &o) {
      bbh_weights_free(handle);
      handle = std::exchange(o.handle, nullptr);
    }
    return *this;
  }
  ~ModelWeights() { bbh_weights_free(handle); }
};

inline ModelWeights load_model_weights(const char* dir = model::WEIGHTS_DIR, int layers = model::NUM_LAYERS,
                                       int device = 0) {
  bbh_weights* w = nullptr;
  bbh_detail::check(bbh_weights_load(dir, layers, device, &w), "load_model_weights");
  return ModelWeights(w);
}

// The same weights from one blob file (bbh_weights_pack of a weights/ folder).
inline ModelWeights load_model_weights_blob(const char* path, int device = 0) {
  bbh_weights* w = nullptr;
  bbh_detail::check(bbh_weights_load_blob(path, device, &w), "load_model_weights_blob");
  return ModelWeights(w);
}

// Scratch sized once for batch x seq tokens. The device buffers are created on the first
// forward (they are tied to the weights' device and GEMM descriptors).
struct Workspace {
  int batch = 1;
  int seq = model::SEQ_LEN;
  bbh_ws* handle = nullptr;
  const bbh_weights* bound = nullptr;
  Workspace(int b, int s) : batch(b), seq(s) {}
  Workspace(const Workspace&) = delete;
  Workspace& operator=(const Workspace&) = delete;
  Workspace(Workspace&& o) noexcept : batch(o.batch), seq(o.seq), handle(std::exchange(o.handle, nullptr)),
                                      bound(o.bound) {}
  ~Workspace() { bbh_ws_free(handle); }
  bbh_ws* get(const ModelWeights& w) {
    if (!handle) {
      bbh_detail::check(bbh_ws_create(w.handle, batch * seq, batch, seq, &handle), "make_workspace");
      bound = w.handle;
    }
    return handle;
  }
};

inline Workspace make_workspace(int batch = 1, int seq = model::SEQ_LEN) { return Workspace(batch, seq); }

inline void bert_encode(Workspace& ws, const ModelWeights& w, const int32_t* input_ids,
                        const int32_t* token_type_ids, const int32_t* mask, __half* out, int batch = 1,
                        int seq = model::SEQ_LEN, cudaStream_t stream = nullptr) {
  bbh_detail::check(bbh_encode(ws.get(w), w.handle, input_ids, token_type_ids, mask,
                               reinterpret_cast<uint16_t*>(out), batch, seq, stream),
                    "bert_encode");
}

inline void bert_embed(Workspace& ws, const ModelWeights& w, const int32_t* input_ids,
                       const int32_t* token_type_ids, const int32_t* mask, __half* embedding, int batch = 1,
                       int seq = model::SEQ_LEN, cudaStream_t stream = nullptr) {
  bbh_detail::check(bbh_embed(ws.get(w), w.handle, input_ids, token_type_ids, mask,
                              reinterpret_cast<uint16_t*>(embedding), batch, seq, stream),
                    "bert_embed");
}

// Packed variable-length form: ids/types [total_tokens], cu_seqlens [batch + 1] (device).
inline void bert_embed_varlen(Workspace& ws, const ModelWeights& w, const int32_t* input_ids,
                              const int32_t* token_type_ids, const int32_t* cu_seqlens, int batch,
                              int total_tokens, int max_len, __half* embedding, cudaStream_t stream = nullptr) {
  bbh_detail::check(bbh_embed_varlen(ws.get(w), w.handle, input_ids, token_type_ids, cu_seqlens, batch,
                                     total_tokens, max_len, reinterpret_cast<uint16_t*>(embedding), stream),
                    "bert_embed_varlen");
}

// Host corpus driver (the reference's bench/corpus.cu loop as a library call): plan
// length-sorted batches once, then embed this rank's batches from host arrays into host
// memory at corpus rows. Aborts on error like the calls above.
struct CorpusPlan {
  std::vector<int32_t> order, batch_first, batch_rank;
  int n_batches = 0;
};

inline CorpusPlan plan_batches(const std::vector<int32_t>& lengths, int max_batch, int max_tokens, int world = 1) {
  CorpusPlan p;
  const int n = static_cast<int>(lengths.size());
  p.order.resize(lengths.size());
  p.batch_first.resize(lengths.size() + 1);
  p.batch_rank.resize(lengths.size() + 1);
  bbh_detail::check(bbh_plan_batches(lengths.data(), n, max_batch, max_tokens, world, p.order.data(),
                                     p.batch_first.data(), p.batch_rank.data(), &p.n_batches),
                    "plan_batches");
  p.batch_first.resize(size_t(p.n_batches) + 1);
  p.batch_rank.resize(size_t(p.n_batches));
  return p;
}

// ids/types: host arrays of all sentences back to back (types may be null); offsets
// [n+1] host; embedding: host [n, 384] fp16.
inline void embed_corpus(Workspace& ws, const ModelWeights& w, const int32_t* ids, const int32_t* types,
                         const int64_t* offsets, int n, const CorpusPlan& plan, __half* embedding, int rank = 0,
                         cudaStream_t stream = nullptr) {
  bbh_detail::check(bbh_embed_corpus(ws.get(w), w.handle, ids, types, offsets, n, plan.order.data(),
                                     plan.batch_first.data(), plan.batch_rank.data(), plan.n_batches, rank,
                                     reinterpret_cast<uint16_t*>(embedding), stream),
                    "embed_corpus");
}

// bert_embed over consecutive batches of `batch` sentences of a padded host corpus:
// ids/types/mask host [n, seq] (types / mask may be null); embedding host [n, 384] fp16.
inline void embed_padded(Workspace& ws, const ModelWeights& w, const int32_t* ids, const int32_t* types,
                         const int32_t* mask, int n, int seq, int batch, __half* embedding,
                         cudaStream_t stream = nullptr) {
  bbh_detail::check(bbh_embed_padded(ws.get(w), w.handle, ids, types, mask, n, seq, batch,
                                     reinterpret_cast<uint16_t*>(embedding), stream),
                    "embed_padded");
}

// WordPiece tokenization into the packed layout of bert_embed_varlen (host vectors).
struct Tokenized {
  std::vector<int32_t> ids, cu_seqlens;
};

class Vocabulary {
 public:
  explicit Vocabulary(const char* vocab_txt, bool lowercase = true) {
    bbh_detail::check(bbh_vocab_load(vocab_txt, lowercase ? 1 : 0, &v_), "Vocabulary");
  }
  Vocabulary(const Vocabulary&) = delete;
  Vocabulary& operator=(const Vocabulary&) = delete;
  ~Vocabulary() { bbh_vocab_free(v_); }

  Tokenized tokenize(const std::vector<std::string>& texts, int max_len = model::SEQ_LEN) const {
    std::vector<const char*> p(texts.size());
    size_t cap = 16;
    for (size_t i = 0; i < texts.size(); ++i) {
      p[i] = texts[i].c_str();
      cap += texts[i].size() + 2;
    }
    Tokenized t;
    t.cu_seqlens.resize(texts.size() + 1);
    int64_t total = 0;
    for (int attempt = 0; attempt < 2; ++attempt) {
      t.ids.resize(cap);
      const int rc = bbh_tokenize(v_, p.data(), static_cast<int>(texts.size()), max_len, t.ids.data(),
                                  static_cast<int64_t>(cap), t.cu_seqlens.data(), &total);
      if (rc == BBH_OK) break;
      if (rc != BBH_ERR_CAPACITY || attempt) bbh_detail::check(rc, "tokenize");
      cap = static_cast<size_t>(total);
    }
    t.ids.resize(static_cast<size_t>(total));
    return t;
  }

 private:
  bbh_vocab* v_ = nullptr;
};
