/* bbh.h -- C ABI of the B200 MiniLM-BERT sentence-embedding engine (libbbh.so).
 *
 * Drop-in for the hot path of tytrdev/bert-by-hand: bert_embed / bert_encode, the
 * per-tensor fp16 weight files and the allocate-once workspace. Plain pointers and
 * sizes only: token arrays are int32, fp16 tensors are passed as uint16_t bit patterns,
 * streams are cudaStream_t passed as void* (NULL = legacy default stream). All data
 * pointers are DEVICE pointers unless stated otherwise, owned by the caller.
 *
 * Every function returns BBH_OK (0) or a negative BBH_ERR_* code; bbh_last_error()
 * gives the message (per thread). Forward calls are asynchronous on the given stream;
 * input problems only visible on the device (bad token ids, malformed cu_seqlens) are
 * recorded in the workspace's device error word, read by bbh_device_error().
 *
 * Model: MiniLM/BERT encoder, hidden 384, 12 heads x 32, FFN 1536 (erf-GELU),
 * vocab 30522, 512 positions, 2 token types, post-LN eps 1e-12; 6 or 12 layers
 * (reference constants: src/core/model_config.h:7-17, made runtime for the layer count).
 */
#ifndef BBH_H_
#define BBH_H_

#include <stdint.h>

#if defined(__GNUC__)
#define BBH_API __attribute__((visibility("default")))
#else
#define BBH_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define BBH_OK 0
#define BBH_ERR_ARG (-1)         /* null pointer, bad shape or alignment */
#define BBH_ERR_CAPACITY (-2)    /* request exceeds the workspace's capacity */
#define BBH_ERR_CUDA (-3)        /* a CUDA runtime/driver call failed */
#define BBH_ERR_IO (-4)          /* weight file missing or short */
#define BBH_ERR_DEVICE (-5)      /* the device flagged bad input or a timed-out wait */
#define BBH_ERR_UNSUPPORTED (-6) /* no sm_100 device */

#define BBH_HIDDEN 384
#define BBH_MAX_POSITIONS 512

typedef struct bbh_weights bbh_weights;
typedef struct bbh_ws bbh_ws;

/* Last error message of the calling thread ("" if none). */
BBH_API const char* bbh_last_error(void);

/* ---- weights ------------------------------------------------------------------------
 * Replaces ModelWeights / load_model_weights() (src/model/weights.h:15-107). Reads the
 * same files: <dir>/<HF state_dict key>.bin, fp16, nn.Linear (out, in) row-major
 * (written by scripts/dump_weights.py:75-82). Q/K/V are concatenated along the output
 * dimension into one [1152, 384] projection as detail::load_qkv does (weights.h:40-54);
 * everything lives in one device arena. */
BBH_API int bbh_num_tensors(int layers);
BBH_API const char* bbh_tensor_name(int layers, int index);
BBH_API int64_t bbh_tensor_numel(int layers, int index);
BBH_API int bbh_weights_load(const char* dir, int layers, int device, bbh_weights** out);
/* tensors[i] = host pointer to tensor i (fp16 bits) in bbh_tensor_name() order. */
BBH_API int bbh_weights_from_host(const uint16_t* const* tensors, int layers, int device, bbh_weights** out);
/* Single-file weight blob (no counterpart in the reference, which opens one file per
 * tensor): bbh_weights_pack (host only) reads <dir>/<key>.bin for every tensor of the
 * catalogue and writes one file -- header "BBHW", version, layer and tensor counts, data
 * offset/size and an FNV-1a 64 checksum, a table of (name, numel, offset), then the fp16
 * tensors 256-byte aligned. bbh_blob_check (host only) validates a blob (magic, version,
 * names and sizes against the catalogue, bounds, checksum) and returns its layer count;
 * bbh_weights_load_blob loads it into a device arena with one read (BBH_ERR_IO on any
 * mismatch or corruption). */
BBH_API int bbh_weights_pack(const char* dir, int layers, const char* blob_path);
BBH_API int bbh_blob_check(const char* blob_path, int* layers);
BBH_API int bbh_weights_load_blob(const char* blob_path, int device, bbh_weights** out);
BBH_API void bbh_weights_free(bbh_weights* w);
BBH_API int bbh_weights_layers(const bbh_weights* w);

/* ---- workspace ----------------------------------------------------------------------
 * Replaces Workspace / make_workspace(batch) (src/model/workspace.h:10-36): every
 * activation buffer is allocated once, for max_tokens rows (padded: batch*seq; packed:
 * total real tokens), max_batch sentences and sentences of at most max_len tokens.
 * Unlike the reference, requests beyond the capacity are rejected with
 * BBH_ERR_CAPACITY instead of overflowing. One workspace per concurrent stream. */
BBH_API int bbh_ws_create(const bbh_weights* w, int max_tokens, int max_batch, int max_len, bbh_ws** out);
BBH_API void bbh_ws_free(bbh_ws* ws);
/* 1 (default): the forward's kernels launch with programmatic dependent launch -- each
 * kernel lets the next one start its launch and prologue (barrier set-up, tensor-memory
 * allocation, weight staging) while it finishes, and the next one waits for its results
 * before touching them; 0: plain stream order. Results are identical either way. */
BBH_API int bbh_ws_set_pdl(bbh_ws* ws, int enable);
/* GEMM tile shape: 0 = one SM per 128-row tile; 1 = pairs of SMs sharing one 256-row tile
 * (tcgen05 cta_group::2), 192 columns wide where N allows, else 256; 2 (default) = pairs,
 * 256 columns first (the first FFN layer, N = 1536; QKV, N = 1152, stays at 192). In modes
 * 1 and 2 the residual-LayerNorm GEMMs give each SM pair a whole 256 x 384 tile. All modes
 * give bit-identical results.
 * bbh_ws_set_gemm_pairs sets it for one workspace (its plans are rebuilt by the next
 * forward; not while a forward of that workspace is being enqueued on another thread).
 * bbh_set_gemm_pairs sets the process-wide default (an atomic value) that workspaces
 * created afterwards and the unit operators (bbh_linear*) use. No reference counterpart:
 * the reference has one wmma tile shape (src/kernels/matmul.cu:64-92). */
BBH_API int bbh_ws_set_gemm_pairs(bbh_ws* ws, int mode);
BBH_API int bbh_set_gemm_pairs(int mode);
/* 1: every kernel of this workspace's forwards carries an L2 access-policy window over the
 * encoder layers' weights (hits persist, misses stream), and the process's persisting-L2
 * set-aside is raised to the window's size (cudaLimitPersistingL2CacheSize; a setting of this
 * process's CUDA context that ends with it). 0 (default): no window. Needs the weights the
 * workspace was created with. The reference keeps its weights in 101 separate buffers with
 * no cache policy (src/model/weights.h:86-107). */
BBH_API int bbh_ws_set_l2_persist(bbh_ws* ws, int enable);
/* 1 (default): bbh_embed* replay one captured CUDA graph per workspace; 0: eager launches. */
BBH_API int bbh_ws_set_graph(bbh_ws* ws, int enable);
/* Synchronises the device, returns the workspace's device error code (0 = none) and
 * optionally clears it. */
BBH_API int bbh_device_error(bbh_ws* ws, int reset);
/* Number of kernel launches one forward of this workspace's model issues. */
BBH_API int bbh_launches_per_forward(const bbh_ws* ws);
/* Per-kernel timing (the reference's Timer, src/core/timer.h:6-49, per kernel): while
 * enabled, forwards run as eager launches with a CUDA event pair around every kernel.
 * bbh_ws_kernel_times synchronises, adds the elapsed milliseconds and launch counts per
 * kernel kind into ms[BBH_KERNEL_KINDS] / counts[BBH_KERNEL_KINDS] and resets them.
 * Kinds: 0 embed+LN, 1 QKV GEMM, 2 attention, 3 O GEMM+LN, 4 FFN1 GEMM+GELU,
 * 5 FFN2 GEMM+LN, 6 pool+L2. */
#define BBH_KERNEL_KINDS 7
BBH_API int bbh_ws_set_kernel_timing(bbh_ws* ws, int enable);
BBH_API int bbh_ws_kernel_times(bbh_ws* ws, double* ms, int64_t* counts);

/* ---- forward ------------------------------------------------------------------------
 * bert_embed (src/model/forward.h:17-19, forward.cu:44-53): ids/types/mask are
 * [batch, seq] int32 row-major (padded layout, position = row % seq); emb is
 * [batch, 384] fp16, unit L2 norm, 16-byte aligned (rows are written as 16-byte pieces;
 * BBH_ERR_ARG otherwise). types may be NULL (all 0), mask may be NULL (all 1).
 * seq may be any value in [1, 512] (no multiple-of-16 requirement). */
BBH_API int bbh_embed(bbh_ws* ws, const bbh_weights* w, const int32_t* ids, const int32_t* types, const int32_t* mask,
              uint16_t* emb, int batch, int seq, void* stream);
/* bert_encode (src/model/forward.h:11-13, forward.cu:20-42): final hidden states
 * [batch*seq, 384] fp16 into out. */
BBH_API int bbh_encode(bbh_ws* ws, const bbh_weights* w, const int32_t* ids, const int32_t* types, const int32_t* mask,
               uint16_t* out, int batch, int seq, void* stream);
/* Packed variable-length form (no counterpart in the reference, which only pads):
 * ids/types are [total_tokens] (sentences back to back), cu_seqlens [batch+1] device
 * int32 offsets with cu_seqlens[0] = 0 and cu_seqlens[batch] = total_tokens; max_len
 * bounds every sentence length. emb is [batch, 384] fp16, 16-byte aligned. */
BBH_API int bbh_embed_varlen(bbh_ws* ws, const bbh_weights* w, const int32_t* ids, const int32_t* types,
                     const int32_t* cu_seqlens, int batch, int total_tokens, int max_len, uint16_t* emb,
                     void* stream);
/* Packed encode: out [total_tokens, 384]. layer_dump (may be NULL) receives the hidden
 * state after the embedding LayerNorm and after each layer: [(layers+1), total_tokens, 384]. */
BBH_API int bbh_encode_varlen(bbh_ws* ws, const bbh_weights* w, const int32_t* ids, const int32_t* types,
                      const int32_t* cu_seqlens, int batch, int total_tokens, int max_len, uint16_t* out,
                      uint16_t* layer_dump, void* stream);

/* Parity aid: runs only the forward's first kernel (embedding gather + LayerNorm) and writes,
 * per token t, indices[4t .. 4t+3] = (word id, position id, type id, mask) -- the rows the
 * gather reads and whether the token attends / is pooled -- so a test can compare them with
 * the reference's indexing for equality (src/kernels/embedding.cu:20-25: position = row %
 * seq in the padded layout; src/kernels/pooling.cu:23-28: pooled where mask != 0). Packed
 * when cu_seqlens is non-null (batch, total_tokens, max_len as bbh_embed_varlen; positions
 * restart at 0 in each sentence), else padded (batch, seq, mask as bbh_embed). indices:
 * device int32 [T, 4], 16-byte aligned. */
BBH_API int bbh_embed_gather_indices(bbh_ws* ws, const bbh_weights* w, const int32_t* ids, const int32_t* types,
                                     const int32_t* mask, const int32_t* cu_seqlens, int batch, int seq,
                                     int total_tokens, int max_len, int32_t* indices, void* stream);

/* ---- unit operators (the reference's launch_* kernel API) ---------------------------- */
/* launch_matmul (src/kernels/matmul.h): C[M,N] = A[M,K] W[N,K]^T (+ bias) (+ erf-GELU).
 * N, K multiples of 8; 16-byte aligned pointers. fp16 operands, fp32 accumulation (the
 * reference accumulates in fp16). The GELU is erf-GELU evaluated as x/2 (1 + tanh(y(x)))
 * with y a fitted odd polynomial on the fp16-rounded GEMM output: max abs error ~1.5e-3
 * against the exact erf form (about one fp16 ulp of the output), x or 0 beyond |x| = 5.5. */
BBH_API int bbh_linear(const uint16_t* A, const uint16_t* W, const uint16_t* bias, uint16_t* C, int M, int N, int K,
               int gelu, void* stream);
/* matmul + residual LayerNorm fused (encoder.cu:47-50 / 61-64): C = LN(A W^T + bias +
 * residual) * gamma + beta, N = 384. */
BBH_API int bbh_linear_residual_layernorm(const uint16_t* A, const uint16_t* W, const uint16_t* bias,
                                  const uint16_t* residual, const uint16_t* gamma, const uint16_t* beta, float eps,
                                  uint16_t* C, int M, int K, void* stream);
/* launch_layernorm (src/kernels/layernorm.h): y = LN(x [+ residual]); D must be 384. */
BBH_API int bbh_layernorm(const uint16_t* x, const uint16_t* gamma, const uint16_t* beta, uint16_t* y, int M, int D,
                  float eps, const uint16_t* residual, void* stream);
/* launch_attention_scores + launch_softmax + launch_attention_context
 * (src/kernels/attention.h, softmax.h): qkv [T, 1152] -> ctx [T, 384], sentences given
 * by cu_seqlens [batch+1] (device); keymask [T] uint8 (device, NULL = all keys valid). */
BBH_API int bbh_attention_varlen(const uint16_t* qkv, uint16_t* ctx, const int32_t* cu_seqlens, const uint8_t* keymask,
                         int batch, int max_len, void* stream);
/* launch_mean_pool + launch_l2_normalize (src/kernels/pooling.h, normalize.h) over
 * packed segments: hidden [T, 384] -> emb [batch, 384] (both 16-byte aligned); tokmask as
 * above. */
BBH_API int bbh_mean_pool_l2(const uint16_t* hidden, const int32_t* cu_seqlens, const uint8_t* tokmask, int batch,
                     uint16_t* emb, void* stream);

/* ---- host corpus driver --------------------------------------------------------------
 * The reference's corpus loop (bench/corpus.cu:80-160) as a library call: sort the
 * sentences by length, cut batches, run them, gather the embeddings back to corpus order.
 *
 * bbh_plan_batches (host only, no GPU needed): lengths [n] (host). Stable sort by
 * length into order [n] (corpus indices); batches are consecutive runs of order[] with at
 * most max_batch sentences and max_tokens tokens: batch b is order[batch_first[b] ..
 * batch_first[b+1]), batch_first has room for n+1 entries. batch_rank [n] receives the
 * rank of each batch for `world` ranks, by longest-processing-time first on each batch's
 * FLOPs (sum over its sentences of 3,538,944 L + 1,536 L^2), so ranks finish together.
 * *n_batches receives the batch count. A sentence longer than max_tokens or 512 returns
 * BBH_ERR_CAPACITY. */
BBH_API int bbh_plan_batches(const int32_t* lengths, int n, int max_batch, int max_tokens, int world, int32_t* order,
                             int32_t* batch_first, int32_t* batch_rank, int* n_batches);
/* bbh_embed_corpus: runs the batches of a plan that belong to `rank` and writes their
 * sentences' embeddings into emb [n, 384] fp16 at their corpus rows (other rows are not
 * touched). ids/types (types may be NULL = all 0) are HOST arrays of all sentences back
 * to back, sentence i = [offsets[i], offsets[i+1]) (HOST int64 [n+1]); emb is HOST
 * memory. Each batch is gathered into one of two pinned staging slots, copied to the
 * device on a copy stream, embedded on `stream` (one graph replay), and copied back on a
 * second copy stream, so the staging of one batch overlaps the forward of the previous
 * one. Returns when every result is in emb. Batches must fit the workspace (checked on the
 * host before anything runs); device-detected input errors return BBH_ERR_DEVICE. */
/* Compute lanes of bbh_embed_corpus for this workspace: 1 (default) or 2. With 2 the driver
 * creates (on first use, freed with ws) a second workspace of the same capacity and a
 * second compute stream, and alternates batches between them so that neighbouring
 * forwards overlap on the GPU (short-sentence corpora gain the most). */
BBH_API int bbh_ws_set_corpus_lanes(bbh_ws* ws, int lanes);
BBH_API int bbh_embed_corpus(bbh_ws* ws, const bbh_weights* w, const int32_t* ids, const int32_t* types,
                             const int64_t* offsets, int n, const int32_t* order, const int32_t* batch_first,
                             const int32_t* batch_rank, int n_batches, int rank, uint16_t* emb, void* stream);
/* bbh_embed_corpus_device: the same loop with the embeddings left in DEVICE memory for a
 * collective to gather: emb_dev [m, 384] fp16 (16-byte aligned) receives the m sentences of
 * this rank's batches in plan order (batch after batch, each batch's sentences in
 * order[batch_first[b] .. batch_first[b+1])), so rank r's rows map to corpus rows through
 * the plan. No device->host copy. Returns when every result is in emb_dev. Replaces the
 * per-batch bert_embed loop of bench/corpus.cu:118-128 for a multi-GPU caller. */
BBH_API int bbh_embed_corpus_device(bbh_ws* ws, const bbh_weights* w, const int32_t* ids, const int32_t* types,
                                    const int64_t* offsets, int n, const int32_t* order, const int32_t* batch_first,
                                    const int32_t* batch_rank, int n_batches, int rank, uint16_t* emb_dev,
                                    void* stream);

/* bbh_embed_padded: bert_embed (the call the reference's bench/bench.cu:44-49 repeats on
 * device-resident inputs) over consecutive batches of a padded [n, seq] corpus held in host
 * memory, as one call. ids/types/mask are
 * HOST int32 [n, seq] row-major (types / mask may be NULL: all 0 / all 1); batches of
 * `batch` consecutive sentences (the last may be shorter) go through the same two pinned
 * staging slots, copy streams and lanes as bbh_embed_corpus; emb is HOST fp16 [n, 384].
 * batch x seq must fit the workspace (BBH_ERR_CAPACITY otherwise). */
BBH_API int bbh_embed_padded(bbh_ws* ws, const bbh_weights* w, const int32_t* ids, const int32_t* types,
                             const int32_t* mask, int n, int seq, int batch, uint16_t* emb, void* stream);

/* ---- the step before the path: WordPiece tokenizer (host only) ---------------------------
 * The reference tokenizes with the HF tokenizer of its sentence-transformers model
 * (scripts/dump_corpus.py:34-38: BERT uncased, truncation=True, max_length=128) and has no
 * tokenizer of its own. bbh_vocab_load reads a BERT vocab.txt (one token per line, id =
 * line number; must contain [UNK], [CLS], [SEP]); lowercase = 1 for uncased models (also
 * strips accents). bbh_tokenize turns n UTF-8 texts into the packed layout of
 * bbh_embed_varlen: ids[total] = [CLS] pieces [SEP] per text, each text truncated to
 * max_len tokens including the two specials, cu_seqlens[n+1] offsets (host arrays).
 * *total receives the number of ids; if it exceeds ids_cap nothing past ids_cap is written
 * and BBH_ERR_CAPACITY is returned (call again with a larger buffer). */
typedef struct bbh_vocab bbh_vocab;
BBH_API int bbh_vocab_load(const char* vocab_path, int lowercase, bbh_vocab** out);
BBH_API void bbh_vocab_free(bbh_vocab* v);
BBH_API int bbh_vocab_size(const bbh_vocab* v);
BBH_API int bbh_tokenize(const bbh_vocab* v, const char* const* texts, int n, int max_len, int32_t* ids,
                         int64_t ids_cap, int32_t* cu_seqlens, int64_t* total);

/* ---- the step after the path: similarity evaluation -----------------------------------
 * scripts/benchmark.py:54-61 of the reference: sims = einsum("ij,ij->i", embs[a], embs[b])
 * over sentence pairs, then scipy's spearmanr against gold scores.
 * bbh_pair_similarity: emb [n, 384] fp16 (device, 16-byte aligned), pairs [m, 2] int32
 * (device) -> sims [m] fp32 (device), dot products in fp32 (the cosine for unit
 * embeddings). A pair with an index outside [0, n) gives NaN. Asynchronous on stream.
 * bbh_spearman (host only): Spearman rank correlation of x and y [n] (ties get average
 * ranks, as scipy.stats.spearmanr); n >= 2, no NaN. */
BBH_API int bbh_pair_similarity(const uint16_t* emb, int n, const int32_t* pairs, int m, float* sims, void* stream);
BBH_API int bbh_spearman(const float* x, const float* y, int n, double* rho);

/* ---- forward without device allocation ----------------------------------------------
 * No counterpart in the reference. Some callers cannot call cudaMalloc: hosts whose own
 * pool allocator owns all device memory and forbids allocations behind its back, and
 * latency-critical paths that cannot take the implicit device synchronisation a
 * cudaMalloc may cause. This variant of bbh_embed_varlen allocates nothing: its scratch
 * (activations, sentence table, error word) lives in one fixed array of device memory
 * inside libbbh.so, about 7.5 MB, which every GPU that loads the library keeps until the
 * process exits. The caller still passes the weights, inputs and output.
 * Limits: total_tokens <= BBH_STATIC_MAX_TOKENS, batch <= BBH_STATIC_MAX_BATCH,
 * max_len <= 512; larger requests return BBH_ERR_CAPACITY with a message saying so.
 * The first call on each device looks up the array's device address (a
 * cudaGetSymbolAddress with that device current), so make that first call before any
 * stream capture. The GEMM tensor maps are encoded on the host on the first call with a
 * given weight set and reused while later calls pass the same one. All calls share the one array and it keeps the last call's contents:
 * calls that overlap on the GPU (for example on two streams of the same device) race and
 * corrupt each other's results, so serialise them. Device-side input errors go to the
 * array's own error word, cleared at the start of each call; read it with
 * bbh_static_device_error(). */
#define BBH_STATIC_MAX_TOKENS 1024
#define BBH_STATIC_MAX_BATCH 128
BBH_API int bbh_embed_varlen_static(const bbh_weights* w, const int32_t* ids, const int32_t* types,
                                    const int32_t* cu_seqlens, int batch, int total_tokens, int max_len,
                                    uint16_t* emb, void* stream);
/* Synchronises the current device and returns the static path's device error code. */
BBH_API int bbh_static_device_error(void);

#ifdef __cplusplus
}
#endif

#endif /* BBH_H_ */
