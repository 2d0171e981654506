// Host corpus driver: length bucketing, rank assignment and a pipelined host -> device ->
// host loop around the packed forward. Replaces the corpus loop of the reference's
// bench/corpus.cu:80-160 (sort by length, cut batches, one bert_embed per batch, gather
// the results back to corpus order), which pads every batch to its longest sentence and
// stages inputs synchronously. Here batches are packed (cu_seqlens), bounded by the
// workspace's token capacity as well as its sentence count, assigned to ranks by
// longest-processing-time on their FLOPs, and run with two staging slots so the host
// gather, the host->device copy, the forward and the device->host copy of neighbouring
// batches overlap. With two lanes (bbh_ws_set_corpus_lanes) alternate batches also run on a
// second workspace and compute stream, so neighbouring forwards overlap on the GPU.
#include "internal.h"
#include "../../include/bbh.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <numeric>
#include <string>
#include <vector>

namespace {

// GEMM + attention FLOPs of one sentence of L tokens per layer (the layer count is a
// common factor and does not change the assignment).
double sentence_work(int64_t L) { return 3538944.0 * double(L) + 1536.0 * double(L) * double(L); }

struct Slot {
  int32_t *h_ids = nullptr, *h_types = nullptr, *h_cu = nullptr, *h_mask = nullptr;  // pinned
  uint16_t* h_emb = nullptr;                                                         // pinned
  int32_t *d_ids = nullptr, *d_types = nullptr, *d_cu = nullptr, *d_mask = nullptr;
  uint16_t* d_emb = nullptr;
  cudaEvent_t h2d = nullptr, fwd = nullptr, d2h = nullptr;
  int batch = -1;  // plan batch whose results the slot holds (-1: none)
};

struct Stage {
  int device = 0;
  int max_tokens = 0, max_batch = 0;
  cudaStream_t up = nullptr, down = nullptr;  // host->device, device->host copy streams
  Slot slot[2];
  // second lane: a workspace of the same capacity and its own compute stream, so that the
  // forwards of neighbouring batches can overlap (one batch's kernel tails and launch
  // gaps are filled with the other's work)
  int lanes = 1;
  bbh_ws* ws2 = nullptr;
  cudaStream_t s2 = nullptr;
};

void free_stage(void* p) {
  Stage* st = static_cast<Stage*>(p);
  if (!st) return;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(st->device);
  for (Slot& s : st->slot) {
    if (s.h2d) cudaEventSynchronize(s.h2d);
    if (s.d2h) cudaEventSynchronize(s.d2h);
    cudaFreeHost(s.h_ids);
    cudaFreeHost(s.h_types);
    cudaFreeHost(s.h_cu);
    cudaFreeHost(s.h_mask);
    cudaFreeHost(s.h_emb);
    cudaFree(s.d_ids);
    cudaFree(s.d_types);
    cudaFree(s.d_cu);
    cudaFree(s.d_mask);
    cudaFree(s.d_emb);
    for (cudaEvent_t e : {s.h2d, s.fwd, s.d2h})
      if (e) cudaEventDestroy(e);
  }
  if (st->s2) cudaStreamSynchronize(st->s2);
  if (st->ws2) bbh_ws_free(st->ws2);
  if (st->s2) cudaStreamDestroy(st->s2);
  if (st->up) cudaStreamDestroy(st->up);
  if (st->down) cudaStreamDestroy(st->down);
  cudaSetDevice(prev);
  delete st;
}

int make_stage(bbh_ws* ws, Stage** out) {
  int device = 0, max_tokens = 0, max_batch = 0, max_len = 0;
  bbh::ws_limits(ws, &device, &max_tokens, &max_batch, &max_len);
  Stage* st = new Stage;
  st->device = device;
  st->max_tokens = max_tokens;
  st->max_batch = max_batch;
  bool ok = cudaStreamCreateWithFlags(&st->up, cudaStreamNonBlocking) == cudaSuccess &&
            cudaStreamCreateWithFlags(&st->down, cudaStreamNonBlocking) == cudaSuccess;
  const size_t tok = size_t(max_tokens) * sizeof(int32_t);
  const size_t cu = size_t(max_batch + 1) * sizeof(int32_t);
  const size_t emb = size_t(max_batch) * BBH_HIDDEN * sizeof(uint16_t);
  for (Slot& s : st->slot) {
    ok = ok && cudaHostAlloc(&s.h_ids, tok, cudaHostAllocDefault) == cudaSuccess &&
         cudaHostAlloc(&s.h_types, tok, cudaHostAllocDefault) == cudaSuccess &&
         cudaHostAlloc(&s.h_cu, cu, cudaHostAllocDefault) == cudaSuccess &&
         cudaHostAlloc(&s.h_mask, tok, cudaHostAllocDefault) == cudaSuccess &&
         cudaHostAlloc(&s.h_emb, emb, cudaHostAllocDefault) == cudaSuccess &&
         cudaMalloc(&s.d_ids, tok) == cudaSuccess && cudaMalloc(&s.d_types, tok) == cudaSuccess &&
         cudaMalloc(&s.d_cu, cu) == cudaSuccess && cudaMalloc(&s.d_mask, tok) == cudaSuccess &&
         cudaMalloc(&s.d_emb, emb) == cudaSuccess &&
         cudaEventCreateWithFlags(&s.h2d, cudaEventDisableTiming) == cudaSuccess &&
         cudaEventCreateWithFlags(&s.fwd, cudaEventDisableTiming) == cudaSuccess &&
         cudaEventCreateWithFlags(&s.d2h, cudaEventDisableTiming) == cudaSuccess;
  }
  if (!ok) {
    cudaGetLastError();
    free_stage(st);
    return bbh::internal_fail(BBH_ERR_CUDA, "bbh_embed_corpus: staging allocation failed");
  }
  *out = st;
  return BBH_OK;
}

// The workspace's staging (created on first use, freed with the workspace) and, for two
// lanes, its second workspace and stream. Switches to the workspace's device; *prev gets
// the caller's.
int acquire_stage(bbh_ws* ws, const bbh_weights* w, Stage** out, int* prev, const char* who) {
  int device = 0, max_tokens = 0, max_batch = 0, max_len = 0;
  bbh::ws_limits(ws, &device, &max_tokens, &max_batch, &max_len);
  cudaGetDevice(prev);
  if (cudaSetDevice(device) != cudaSuccess) return bbh::internal_fail(BBH_ERR_CUDA, std::string(who) + ": cudaSetDevice");
  void** slotp = bbh::ws_corpus_stage(ws, free_stage);
  if (!*slotp) {
    Stage* st = nullptr;
    int rc = make_stage(ws, &st);
    if (rc) return rc;
    *slotp = st;
  }
  Stage& st = *static_cast<Stage*>(*slotp);
  if (bbh::ws_corpus_lanes(ws) == 2 && !st.ws2) {
    int rc = bbh_ws_create(w, max_tokens, max_batch, max_len, &st.ws2);
    if (!rc && cudaStreamCreateWithFlags(&st.s2, cudaStreamNonBlocking) != cudaSuccess)
      rc = bbh::internal_fail(BBH_ERR_CUDA, std::string(who) + ": stream creation failed");
    if (rc) return rc;
  }
  if (st.ws2) bbh::ws_inherit_settings(st.ws2, ws);
  *out = &st;
  return BBH_OK;
}

// Device-detected input errors of the workspace(s) after a driver run.
int device_status(bbh_ws* ws, const Stage& st, const char* who) {
  int dev_err = bbh_device_error(ws, 0);
  if (dev_err == 0 && st.ws2) dev_err = bbh_device_error(st.ws2, 0);
  if (dev_err < 0) return dev_err;
  if (dev_err > 0)
    return bbh::internal_fail(BBH_ERR_DEVICE, std::string(who) + ": the device flagged bad input (code " +
                                                  std::to_string(dev_err) + ")");
  return BBH_OK;
}

}  // namespace

extern "C" {

int bbh_plan_batches(const int32_t* lengths, int n, int max_batch, int max_tokens, int world, int32_t* order,
                     int32_t* batch_first, int32_t* batch_rank, int* n_batches) {
  if (n < 0 || max_batch <= 0 || max_tokens <= 0 || world <= 0 || !n_batches || (n > 0 && !lengths) ||
      (n > 0 && (!order || !batch_first || !batch_rank)) || !batch_first)
    return bbh::internal_fail(BBH_ERR_ARG, "bbh_plan_batches: bad arguments");
  for (int i = 0; i < n; ++i) {
    if (lengths[i] < 0) return bbh::internal_fail(BBH_ERR_ARG, "bbh_plan_batches: negative sentence length");
    if (lengths[i] > max_tokens || lengths[i] > BBH_MAX_POSITIONS)
      return bbh::internal_fail(BBH_ERR_CAPACITY, "bbh_plan_batches: sentence " + std::to_string(i) + " has " +
                                                      std::to_string(lengths[i]) +
                                                      " tokens, more than max_tokens or 512 positions");
  }
  // Stable length sort (bench/corpus.cu:87-90 sorts by length; stable keeps ties in corpus
  // order so the plan is deterministic).
  std::vector<int32_t> idx(static_cast<size_t>(n));
  std::iota(idx.begin(), idx.end(), 0);
  std::stable_sort(idx.begin(), idx.end(), [&](int32_t a, int32_t b) { return lengths[a] < lengths[b]; });
  // Consecutive runs of at most max_batch sentences and max_tokens tokens.
  std::vector<int32_t> first;
  std::vector<double> work;
  int64_t tokens = 0;
  int count = 0;
  for (int i = 0; i < n; ++i) {
    const int L = lengths[idx[size_t(i)]];
    if (count == 0 || count == max_batch || tokens + L > max_tokens) {
      first.push_back(i);
      work.push_back(0.0);
      tokens = 0;
      count = 0;
    }
    tokens += L;
    ++count;
    work.back() += sentence_work(L);
  }
  const int nb = static_cast<int>(first.size());
  // Longest processing time first: heaviest batch to the least-loaded rank (ties: lower
  // batch index first, lower rank first).
  std::vector<int32_t> by_work(static_cast<size_t>(nb));
  std::iota(by_work.begin(), by_work.end(), 0);
  std::stable_sort(by_work.begin(), by_work.end(), [&](int32_t a, int32_t b) { return work[a] > work[b]; });
  std::vector<double> load(static_cast<size_t>(world), 0.0);
  for (int32_t b : by_work) {
    const int r = static_cast<int>(std::min_element(load.begin(), load.end()) - load.begin());
    batch_rank[b] = r;
    load[size_t(r)] += work[size_t(b)];
  }
  for (int i = 0; i < n; ++i) order[i] = idx[size_t(i)];
  for (int b = 0; b < nb; ++b) batch_first[b] = first[size_t(b)];
  batch_first[nb] = n;
  *n_batches = nb;
  return BBH_OK;
}

}  // extern "C"

namespace {

// The corpus loop of bbh_embed_corpus (emb: host rows in corpus order) and of
// bbh_embed_corpus_device (emb_dev: device rows, this rank's sentences in plan order).
int corpus_run(const char* who, bbh_ws* ws, const bbh_weights* w, const int32_t* ids, const int32_t* types,
               const int64_t* offsets, int n, const int32_t* order, const int32_t* batch_first,
               const int32_t* batch_rank, int n_batches, int rank, uint16_t* emb, uint16_t* emb_dev, void* stream) {
  const std::string name(who);
  if (!ws || !w || !offsets || n < 0 || n_batches < 0 || !batch_first || (n_batches > 0 && (!order || !batch_rank)) ||
      (n > 0 && (!ids || (!emb && !emb_dev))))
    return bbh::internal_fail(BBH_ERR_ARG, name + ": bad arguments");
  if (emb_dev && (reinterpret_cast<uintptr_t>(emb_dev) & 15))
    return bbh::internal_fail(BBH_ERR_ARG, name + ": the device output must be 16-byte aligned");
  if (batch_first[0] != 0 || batch_first[n_batches] != n)
    return bbh::internal_fail(BBH_ERR_ARG, name + ": batch_first must run from 0 to n");
  int device = 0, max_tokens = 0, max_batch = 0, max_len = 0;
  bbh::ws_limits(ws, &device, &max_tokens, &max_batch, &max_len);
  // validate this rank's batches on the host before anything is queued (other ranks'
  // batches may need more capacity than this rank's workspace has)
  for (int b = 0; b < n_batches; ++b) {
    if (batch_rank[b] != rank) continue;
    const int lo = batch_first[b], hi = batch_first[b + 1];
    if (hi < lo || hi - lo > max_batch)
      return bbh::internal_fail(BBH_ERR_CAPACITY, name + ": batch " + std::to_string(b) +
                                                      " exceeds the workspace's sentence capacity");
    int64_t tok = 0;
    for (int i = lo; i < hi; ++i) {
      const int s = order[i];
      if (s < 0 || s >= n) return bbh::internal_fail(BBH_ERR_ARG, name + ": order out of range");
      const int64_t L = offsets[s + 1] - offsets[s];
      if (L < 0 || L > max_len)
        return bbh::internal_fail(BBH_ERR_CAPACITY, name + ": sentence " + std::to_string(s) +
                                                        " is longer than the workspace's max_len");
      tok += L;
    }
    if (tok > max_tokens)
      return bbh::internal_fail(BBH_ERR_CAPACITY, name + ": batch " + std::to_string(b) +
                                                      " exceeds the workspace's token capacity");
  }
  int prev = 0;
  Stage* stp = nullptr;
  {
    const int rc0 = acquire_stage(ws, w, &stp, &prev, who);
    if (rc0) {
      cudaSetDevice(prev);
      return rc0;
    }
  }
  Stage& st = *stp;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int lanes = bbh::ws_corpus_lanes(ws);

  // Copies a finished slot's embeddings to their corpus rows (host output), or waits until
  // the slot's forward has read its inputs (device output).
  auto drain = [&](Slot& sl) -> int {
    if (sl.batch < 0) return BBH_OK;
    if (emb_dev) {
      sl.batch = -1;
      if (cudaEventSynchronize(sl.fwd) != cudaSuccess)
        return bbh::internal_fail(BBH_ERR_CUDA, name + ": forward failed");
      return BBH_OK;
    }
    if (cudaEventSynchronize(sl.d2h) != cudaSuccess)
      return bbh::internal_fail(BBH_ERR_CUDA, name + ": device->host copy failed");
    const int lo = batch_first[sl.batch], hi = batch_first[sl.batch + 1];
    for (int i = lo; i < hi; ++i)
      std::memcpy(emb + size_t(order[i]) * BBH_HIDDEN, sl.h_emb + size_t(i - lo) * BBH_HIDDEN,
                  BBH_HIDDEN * sizeof(uint16_t));
    sl.batch = -1;
    return BBH_OK;
  };

  int rc = BBH_OK;
  int k = 0;
  size_t dev_row = 0;  // device output: next row of this rank's plan-order embeddings
  for (int b = 0; b < n_batches && rc == BBH_OK; ++b) {
    if (batch_rank[b] != rank) continue;
    Slot& sl = st.slot[k & 1];
    // lane of this batch: its workspace and compute stream
    bbh_ws* lws = (lanes == 2 && (k & 1)) ? st.ws2 : ws;
    cudaStream_t ls = (lanes == 2 && (k & 1)) ? st.s2 : s;
    ++k;
    rc = drain(sl);  // also guarantees the slot's buffers are no longer in use
    if (rc) break;
    const int lo = batch_first[b], hi = batch_first[b + 1], count = hi - lo;
    if (count == 0) continue;
    // gather the batch's sentences (length-sorted) into the pinned slot
    int32_t tok = 0, blen = 0;
    sl.h_cu[0] = 0;
    for (int i = lo; i < hi; ++i) {
      const int sidx = order[i];
      const int32_t L = static_cast<int32_t>(offsets[sidx + 1] - offsets[sidx]);
      std::memcpy(sl.h_ids + tok, ids + offsets[sidx], size_t(L) * sizeof(int32_t));
      if (types) std::memcpy(sl.h_types + tok, types + offsets[sidx], size_t(L) * sizeof(int32_t));
      tok += L;
      blen = std::max(blen, L);
      sl.h_cu[i - lo + 1] = tok;
    }
    const size_t tb = size_t(tok) * sizeof(int32_t);
    bool ok = cudaMemcpyAsync(sl.d_ids, sl.h_ids, tb, cudaMemcpyHostToDevice, st.up) == cudaSuccess &&
              (!types || cudaMemcpyAsync(sl.d_types, sl.h_types, tb, cudaMemcpyHostToDevice, st.up) == cudaSuccess) &&
              cudaMemcpyAsync(sl.d_cu, sl.h_cu, size_t(count + 1) * sizeof(int32_t), cudaMemcpyHostToDevice, st.up) ==
                  cudaSuccess &&
              cudaEventRecord(sl.h2d, st.up) == cudaSuccess && cudaStreamWaitEvent(ls, sl.h2d, 0) == cudaSuccess;
    if (!ok) {
      rc = bbh::internal_fail(BBH_ERR_CUDA, name + ": host->device copy failed");
      break;
    }
    uint16_t* out = emb_dev ? emb_dev + dev_row * BBH_HIDDEN : sl.d_emb;
    dev_row += size_t(count);
    rc = bbh_embed_varlen(lws, w, sl.d_ids, types ? sl.d_types : nullptr, sl.d_cu, count, tok, std::max(blen, 1),
                          out, ls);
    if (rc) break;
    if (emb_dev) {
      if (cudaEventRecord(sl.fwd, ls) != cudaSuccess) {
        rc = bbh::internal_fail(BBH_ERR_CUDA, name + ": event record failed");
        break;
      }
      sl.batch = b;
      continue;
    }
    ok = cudaEventRecord(sl.fwd, ls) == cudaSuccess && cudaStreamWaitEvent(st.down, sl.fwd, 0) == cudaSuccess &&
         cudaMemcpyAsync(sl.h_emb, sl.d_emb, size_t(count) * BBH_HIDDEN * sizeof(uint16_t), cudaMemcpyDeviceToHost,
                         st.down) == cudaSuccess &&
         cudaEventRecord(sl.d2h, st.down) == cudaSuccess;
    if (!ok) {
      rc = bbh::internal_fail(BBH_ERR_CUDA, name + ": device->host copy failed");
      break;
    }
    sl.batch = b;
  }
  for (Slot& sl : st.slot) {
    const int r2 = drain(sl);
    if (!rc) rc = r2;
    sl.batch = -1;
  }
  if (!rc) rc = device_status(ws, st, who);
  cudaSetDevice(prev);
  return rc;
}

}  // namespace

extern "C" {

int bbh_embed_corpus(bbh_ws* ws, const bbh_weights* w, const int32_t* ids, const int32_t* types,
                     const int64_t* offsets, int n, const int32_t* order, const int32_t* batch_first,
                     const int32_t* batch_rank, int n_batches, int rank, uint16_t* emb, void* stream) {
  if (n > 0 && !emb) return bbh::internal_fail(BBH_ERR_ARG, "bbh_embed_corpus: bad arguments");
  return corpus_run("bbh_embed_corpus", ws, w, ids, types, offsets, n, order, batch_first, batch_rank, n_batches,
                    rank, emb, nullptr, stream);
}

int bbh_embed_corpus_device(bbh_ws* ws, const bbh_weights* w, const int32_t* ids, const int32_t* types,
                            const int64_t* offsets, int n, const int32_t* order, const int32_t* batch_first,
                            const int32_t* batch_rank, int n_batches, int rank, uint16_t* emb_dev, void* stream) {
  if (n > 0 && !emb_dev) return bbh::internal_fail(BBH_ERR_ARG, "bbh_embed_corpus_device: bad arguments");
  return corpus_run("bbh_embed_corpus_device", ws, w, ids, types, offsets, n, order, batch_first, batch_rank,
                    n_batches, rank, nullptr, emb_dev, stream);
}

int bbh_embed_padded(bbh_ws* ws, const bbh_weights* w, const int32_t* ids, const int32_t* types, const int32_t* mask,
                     int n, int seq, int batch, uint16_t* emb, void* stream) {
  if (!ws || !w || n < 0 || seq <= 0 || batch <= 0 || (n > 0 && (!ids || !emb)))
    return bbh::internal_fail(BBH_ERR_ARG, "bbh_embed_padded: bad arguments");
  int device = 0, max_tokens = 0, max_batch = 0, max_len = 0;
  bbh::ws_limits(ws, &device, &max_tokens, &max_batch, &max_len);
  if (batch > max_batch || int64_t(batch) * seq > max_tokens || seq > max_len)
    return bbh::internal_fail(BBH_ERR_CAPACITY, "bbh_embed_padded: batch x seq exceeds the workspace");
  int prev = 0;
  Stage* stp = nullptr;
  {
    const int rc0 = acquire_stage(ws, w, &stp, &prev, "bbh_embed_padded");
    if (rc0) {
      cudaSetDevice(prev);
      return rc0;
    }
  }
  Stage& st = *stp;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int lanes = bbh::ws_corpus_lanes(ws);
  // a slot's results are the consecutive rows [first, first + count) of emb
  int first_of[2] = {0, 0}, count_of[2] = {0, 0};
  auto drain = [&](int k) -> int {
    Slot& sl = st.slot[k];
    if (sl.batch < 0) return BBH_OK;
    if (cudaEventSynchronize(sl.d2h) != cudaSuccess)
      return bbh::internal_fail(BBH_ERR_CUDA, "bbh_embed_padded: device->host copy failed");
    std::memcpy(emb + size_t(first_of[k]) * BBH_HIDDEN, sl.h_emb, size_t(count_of[k]) * BBH_HIDDEN * sizeof(uint16_t));
    sl.batch = -1;
    return BBH_OK;
  };
  int rc = BBH_OK;
  int k = 0;
  for (int b = 0, first = 0; first < n && rc == BBH_OK; ++b, first += batch) {
    const int si = k & 1;
    Slot& sl = st.slot[si];
    bbh_ws* lws = (lanes == 2 && si) ? st.ws2 : ws;
    cudaStream_t ls = (lanes == 2 && si) ? st.s2 : s;
    ++k;
    rc = drain(si);  // also guarantees the slot's buffers are no longer in use
    if (rc) break;
    const int count = std::min(batch, n - first);
    const size_t off = size_t(first) * seq, tb = size_t(count) * seq * sizeof(int32_t);
    std::memcpy(sl.h_ids, ids + off, tb);
    if (types) std::memcpy(sl.h_types, types + off, tb);
    if (mask) std::memcpy(sl.h_mask, mask + off, tb);
    bool ok = cudaMemcpyAsync(sl.d_ids, sl.h_ids, tb, cudaMemcpyHostToDevice, st.up) == cudaSuccess &&
              (!types || cudaMemcpyAsync(sl.d_types, sl.h_types, tb, cudaMemcpyHostToDevice, st.up) == cudaSuccess) &&
              (!mask || cudaMemcpyAsync(sl.d_mask, sl.h_mask, tb, cudaMemcpyHostToDevice, st.up) == cudaSuccess) &&
              cudaEventRecord(sl.h2d, st.up) == cudaSuccess && cudaStreamWaitEvent(ls, sl.h2d, 0) == cudaSuccess;
    if (!ok) {
      rc = bbh::internal_fail(BBH_ERR_CUDA, "bbh_embed_padded: host->device copy failed");
      break;
    }
    rc = bbh_embed(lws, w, sl.d_ids, types ? sl.d_types : nullptr, mask ? sl.d_mask : nullptr, sl.d_emb, count, seq,
                   ls);
    if (rc) break;
    ok = cudaEventRecord(sl.fwd, ls) == cudaSuccess && cudaStreamWaitEvent(st.down, sl.fwd, 0) == cudaSuccess &&
         cudaMemcpyAsync(sl.h_emb, sl.d_emb, size_t(count) * BBH_HIDDEN * sizeof(uint16_t), cudaMemcpyDeviceToHost,
                         st.down) == cudaSuccess &&
         cudaEventRecord(sl.d2h, st.down) == cudaSuccess;
    if (!ok) {
      rc = bbh::internal_fail(BBH_ERR_CUDA, "bbh_embed_padded: device->host copy failed");
      break;
    }
    sl.batch = b;
    first_of[si] = first;
    count_of[si] = count;
  }
  for (int i = 0; i < 2; ++i) {
    const int r2 = drain(i);
    if (!rc) rc = r2;
    st.slot[i].batch = -1;
  }
  if (!rc) rc = device_status(ws, st, "bbh_embed_padded");
  cudaSetDevice(prev);
  return rc;
}

}  // extern "C"
