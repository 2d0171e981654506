"""Python host binding of libbbh.so (ctypes over the C ABI in include/bbh.h).

Mirrors the reference's host API for the embedding path (tytrdev/bert-by-hand
src/model/forward.h:11-19 bert_encode / bert_embed, weights.h load_model_weights,
workspace.h make_workspace) plus the packed variable-length form and the unit
operators (src/kernels/*.h launch_*). PyTorch is used only to own device memory and
to name the current CUDA stream; all compute runs in libbbh.so's kernels.

There is no fallback: if libbbh.so is missing or the device is not sm_100, calls raise.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libbbh.so")
HIDDEN = 384

BBH_OK = 0
ERRORS = {-1: "BBH_ERR_ARG", -2: "BBH_ERR_CAPACITY", -3: "BBH_ERR_CUDA", -4: "BBH_ERR_IO",
          -5: "BBH_ERR_DEVICE", -6: "BBH_ERR_UNSUPPORTED"}
DEVICE_ERRORS = {0: "ok", 1: "wait timeout", 2: "token or type id out of range",
                 3: "malformed cu_seqlens", 4: "sequence longer than the position table"}

_lib = None

_P = ctypes.c_void_p
_I = ctypes.c_int
_SIGS = {
    "bbh_last_error": (ctypes.c_char_p, []),
    "bbh_num_tensors": (_I, [_I]),
    "bbh_tensor_name": (ctypes.c_char_p, [_I, _I]),
    "bbh_tensor_numel": (ctypes.c_int64, [_I, _I]),
    "bbh_weights_load": (_I, [ctypes.c_char_p, _I, _I, ctypes.POINTER(_P)]),
    "bbh_weights_from_host": (_I, [ctypes.POINTER(_P), _I, _I, ctypes.POINTER(_P)]),
    "bbh_weights_pack": (_I, [ctypes.c_char_p, _I, ctypes.c_char_p]),
    "bbh_blob_check": (_I, [ctypes.c_char_p, ctypes.POINTER(_I)]),
    "bbh_weights_load_blob": (_I, [ctypes.c_char_p, _I, ctypes.POINTER(_P)]),
    "bbh_weights_free": (None, [_P]),
    "bbh_weights_layers": (_I, [_P]),
    "bbh_ws_create": (_I, [_P, _I, _I, _I, ctypes.POINTER(_P)]),
    "bbh_ws_free": (None, [_P]),
    "bbh_ws_set_graph": (_I, [_P, _I]),
    "bbh_ws_set_gemm_pairs": (_I, [_P, _I]),
    "bbh_ws_set_l2_persist": (_I, [_P, _I]),
    "bbh_ws_set_pdl": (_I, [_P, _I]),
    "bbh_set_gemm_pairs": (_I, [_I]),
    "bbh_device_error": (_I, [_P, _I]),
    "bbh_launches_per_forward": (_I, [_P]),
    "bbh_ws_set_kernel_timing": (_I, [_P, _I]),
    "bbh_ws_kernel_times": (_I, [_P, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_int64)]),
    "bbh_embed": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _P]),
    "bbh_encode": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _P]),
    "bbh_embed_varlen": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _P, _P]),
    "bbh_encode_varlen": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _P, _P, _P]),
    "bbh_linear": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _P]),
    "bbh_linear_residual_layernorm": (_I, [_P, _P, _P, _P, _P, _P, ctypes.c_float, _P, _I, _I, _P]),
    "bbh_layernorm": (_I, [_P, _P, _P, _P, _I, _I, ctypes.c_float, _P, _P]),
    "bbh_attention_varlen": (_I, [_P, _P, _P, _P, _I, _I, _P]),
    "bbh_mean_pool_l2": (_I, [_P, _P, _P, _I, _P, _P]),
    "bbh_plan_batches": (_I, [_P, _I, _I, _I, _I, _P, _P, _P, ctypes.POINTER(_I)]),
    "bbh_embed_gather_indices": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P, _P]),
    "bbh_embed_corpus": (_I, [_P, _P, _P, _P, _P, _I, _P, _P, _P, _I, _I, _P, _P]),
    "bbh_embed_corpus_device": (_I, [_P, _P, _P, _P, _P, _I, _P, _P, _P, _I, _I, _P, _P]),
    "bbh_embed_padded": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _P, _P]),
    "bbh_ws_set_corpus_lanes": (_I, [_P, _I]),
    "bbh_vocab_load": (_I, [ctypes.c_char_p, _I, ctypes.POINTER(_P)]),
    "bbh_vocab_free": (None, [_P]),
    "bbh_vocab_size": (_I, [_P]),
    "bbh_tokenize": (_I, [_P, _P, _I, _I, _P, ctypes.c_int64, _P, ctypes.POINTER(ctypes.c_int64)]),
    "bbh_pair_similarity": (_I, [_P, _I, _P, _I, _P, _P]),
    "bbh_spearman": (_I, [_P, _P, _I, ctypes.POINTER(ctypes.c_double)]),
    "bbh_embed_varlen_static": (_I, [_P, _P, _P, _P, _I, _I, _I, _P, _P]),
    "bbh_static_device_error": (_I, []),
}


class BBHError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{ERRORS.get(code, code)}: {msg}")
        self.code = code


def lib() -> ctypes.CDLL:
    """Load libbbh.so (raises if it was not built: run bert-by-hand_b200/build.py)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python bert-by-hand_b200/build.py`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGS)


def _check(rc: int) -> None:
    if rc != BBH_OK:
        raise BBHError(rc, lib().bbh_last_error().decode())


def _ptr(t):
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("expected a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError("expected a contiguous tensor")
    return ctypes.c_void_p(t.data_ptr())


def _stream(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _i32(t):
    if t is None:
        return None
    if t.dtype != torch.int32:
        raise TypeError("token arrays must be int32")
    return _ptr(t)


def _f16(t):
    if t is None:
        return None
    if t.dtype != torch.float16:
        raise TypeError("expected float16")
    return _ptr(t)


def tensor_names(layers: int = 6) -> list[str]:
    L = lib()
    return [L.bbh_tensor_name(layers, i).decode() for i in range(L.bbh_num_tensors(layers))]


class ModelWeights:
    """Device-resident weights (reference: ModelWeights, src/model/weights.h:15-107)."""

    def __init__(self, handle, layers: int, device: int):
        self.handle = handle
        self.layers = layers
        self.device = device

    @classmethod
    def load(cls, directory: str, layers: int = 6, device: int = 0) -> "ModelWeights":
        """load_model_weights(): reads <directory>/<HF key>.bin fp16 files."""
        h = _P()
        _check(lib().bbh_weights_load(directory.encode(), layers, device, ctypes.byref(h)))
        return cls(h, layers, device)

    @classmethod
    def load_blob(cls, path: str, device: int = 0) -> "ModelWeights":
        """One-file weights written by pack_weights()."""
        h = _P()
        _check(lib().bbh_weights_load_blob(path.encode(), device, ctypes.byref(h)))
        return cls(h, lib().bbh_weights_layers(h), device)

    @classmethod
    def from_numpy(cls, weights: dict, layers: int = 6, device: int = 0) -> "ModelWeights":
        """From a {HF key: fp16 ndarray} dict (the same tensors the .bin files hold)."""
        names = tensor_names(layers)
        keep = [np.ascontiguousarray(weights[n], dtype=np.float16) for n in names]
        arr = (_P * len(names))(*[a.ctypes.data for a in keep])
        h = _P()
        _check(lib().bbh_weights_from_host(arr, layers, device, ctypes.byref(h)))
        return cls(h, layers, device)

    def free(self):
        if self.handle:
            lib().bbh_weights_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Workspace:
    """Allocate-once activation workspace (reference: Workspace, src/model/workspace.h:10-36)."""

    def __init__(self, weights: ModelWeights, max_tokens: int, max_batch: int, max_len: int, graph: bool = True):
        self.weights = weights
        self.max_tokens, self.max_batch, self.max_len = max_tokens, max_batch, max_len
        h = _P()
        _check(lib().bbh_ws_create(weights.handle, max_tokens, max_batch, max_len, ctypes.byref(h)))
        self.handle = h
        self.set_graph(graph)

    def set_graph(self, enable: bool):
        _check(lib().bbh_ws_set_graph(self.handle, 1 if enable else 0))

    def set_corpus_lanes(self, lanes: int):
        """1 or 2 compute lanes for embed_corpus (2: alternate batches on a second workspace)."""
        _check(lib().bbh_ws_set_corpus_lanes(self.handle, lanes))

    def set_pdl(self, enable: bool):
        _check(lib().bbh_ws_set_pdl(self.handle, 1 if enable else 0))

    KERNEL_KINDS = ("embed_ln", "qkv_gemm", "attention", "o_gemm_ln", "ffn1_gemm_gelu", "ffn2_gemm_ln", "pool_l2")

    def set_gemm_pairs(self, mode: int):
        """GEMM tiles of this workspace's forwards: 0 = one SM per 128-row tile, 1 = SM pairs
        (256 x 192 where N allows, else 256 x 256), 2 = SM pairs, 256 x 256 first."""
        _check(lib().bbh_ws_set_gemm_pairs(self.handle, int(mode)))

    def set_l2_persist(self, enable: bool):
        """Forward launches carry an L2 access-policy window over the layer weights (persisting)."""
        _check(lib().bbh_ws_set_l2_persist(self.handle, 1 if enable else 0))

    def set_kernel_timing(self, enable: bool):
        _check(lib().bbh_ws_set_kernel_timing(self.handle, 1 if enable else 0))

    def kernel_times(self) -> dict:
        """{kind: (total ms, launches)} since the last call (synchronises)."""
        ms = (ctypes.c_double * len(self.KERNEL_KINDS))()
        n = (ctypes.c_int64 * len(self.KERNEL_KINDS))()
        _check(lib().bbh_ws_kernel_times(self.handle, ms, n))
        return {k: (ms[i], n[i]) for i, k in enumerate(self.KERNEL_KINDS)}

    @property
    def launches_per_forward(self) -> int:
        return lib().bbh_launches_per_forward(self.handle)

    def device_error(self, reset: bool = True) -> int:
        rc = lib().bbh_device_error(self.handle, 1 if reset else 0)
        if rc < 0:
            _check(rc)
        return rc

    # ---- padded (reference layout) ---------------------------------------------------
    def embed(self, ids, types=None, mask=None, out=None, stream=None):
        """bert_embed: ids/types/mask int32 [B, S] on device -> fp16 [B, 384]."""
        B, S = ids.shape
        out = out if out is not None else torch.empty((B, HIDDEN), dtype=torch.float16, device=ids.device)
        _check(lib().bbh_embed(self.handle, self.weights.handle, _i32(ids), _i32(types), _i32(mask), _f16(out),
                               B, S, _stream(stream)))
        return out

    def encode(self, ids, types=None, mask=None, out=None, stream=None):
        """bert_encode: -> fp16 [B*S, 384] final hidden states."""
        B, S = ids.shape
        out = out if out is not None else torch.empty((B * S, HIDDEN), dtype=torch.float16, device=ids.device)
        _check(lib().bbh_encode(self.handle, self.weights.handle, _i32(ids), _i32(types), _i32(mask), _f16(out),
                                B, S, _stream(stream)))
        return out

    # ---- packed variable length --------------------------------------------------------
    def embed_varlen(self, ids, types, cu_seqlens, max_len: int, out=None, stream=None):
        B = cu_seqlens.numel() - 1
        out = out if out is not None else torch.empty((B, HIDDEN), dtype=torch.float16, device=ids.device)
        _check(lib().bbh_embed_varlen(self.handle, self.weights.handle, _i32(ids), _i32(types), _i32(cu_seqlens),
                                      B, ids.numel(), max_len, _f16(out), _stream(stream)))
        return out

    def encode_varlen(self, ids, types, cu_seqlens, max_len: int, dump_layers: bool = False, stream=None):
        B = cu_seqlens.numel() - 1
        T = ids.numel()
        out = torch.empty((T, HIDDEN), dtype=torch.float16, device=ids.device)
        dump = (torch.empty((self.weights.layers + 1, T, HIDDEN), dtype=torch.float16, device=ids.device)
                if dump_layers else None)
        _check(lib().bbh_encode_varlen(self.handle, self.weights.handle, _i32(ids), _i32(types), _i32(cu_seqlens),
                                       B, T, max_len, _f16(out), _f16(dump), _stream(stream)))
        return (out, dump) if dump_layers else out

    def gather_indices(self, ids, types=None, mask=None, cu_seqlens=None, max_len: int = 0, stream=None):
        """(word id, position, type id, mask) per token, as the embedding kernel resolves them:
        int32 CUDA tensor [T, 4]. Packed when cu_seqlens is given (ids [T]), else padded
        (ids [B, S])."""
        if cu_seqlens is not None:
            T, B, S = ids.shape[0], cu_seqlens.shape[0] - 1, 0
        else:
            B, S = ids.shape
            T = B * S
        out = torch.empty((max(T, 1), 4), dtype=torch.int32, device=ids.device)
        _check(lib().bbh_embed_gather_indices(self.handle, self.weights.handle, _i32(ids), _i32(types), _i32(mask),
                                              _i32(cu_seqlens), B, S, T, max_len, ctypes.c_void_p(out.data_ptr()),
                                              _stream(stream)))
        return out[:T]

    # ---- host corpus -------------------------------------------------------------------
    def embed_corpus(self, ids, types, offsets, plan: "CorpusPlan", rank: int = 0, out=None, stream=None):
        """Runs the plan's batches of `rank` from HOST numpy arrays (ids/types int32 of all
        sentences back to back, offsets int64 [n+1]) with pipelined staging; returns the
        fp16 [n, 384] host array with this rank's sentences filled in (corpus order)."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        types = None if types is None else np.ascontiguousarray(types, dtype=np.int32)
        offsets = np.ascontiguousarray(offsets, dtype=np.int64)
        n = offsets.size - 1
        if out is None:
            out = np.zeros((n, HIDDEN), dtype=np.float16)
        if out.dtype != np.float16 or out.shape != (n, HIDDEN) or not out.flags.c_contiguous:
            raise ValueError("out must be a contiguous float16 [n, 384] host array")
        p = lambda a: None if a is None else a.ctypes.data_as(ctypes.c_void_p)
        _check(lib().bbh_embed_corpus(self.handle, self.weights.handle, p(ids), p(types), p(offsets), n,
                                      p(plan.order), p(plan.batch_first), p(plan.batch_rank), plan.n_batches,
                                      rank, p(out), _stream(stream)))
        return out

    def embed_corpus_device(self, ids, types, offsets, plan: "CorpusPlan", rank: int = 0, out=None, stream=None):
        """The same loop with the embeddings left on the device: returns a CUDA fp16 [m, 384]
        tensor holding the m sentences of `rank`'s batches in plan order (corpus indices:
        plan.rank_order(rank)), ready for a collective."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        types = None if types is None else np.ascontiguousarray(types, dtype=np.int32)
        offsets = np.ascontiguousarray(offsets, dtype=np.int64)
        n = offsets.size - 1
        m = int(plan.rank_order(rank).size)
        if out is None:
            out = torch.empty((max(m, 1), HIDDEN), dtype=torch.float16, device=f"cuda:{self.weights.device}")
        if out.dtype != torch.float16 or out.shape[0] < m or out.shape[1] != HIDDEN or not out.is_contiguous():
            raise ValueError("out must be a contiguous CUDA float16 [>= m, 384] tensor")
        p = lambda a: None if a is None else a.ctypes.data_as(ctypes.c_void_p)
        _check(lib().bbh_embed_corpus_device(self.handle, self.weights.handle, p(ids), p(types), p(offsets), n,
                                             p(plan.order), p(plan.batch_first), p(plan.batch_rank), plan.n_batches,
                                             rank, ctypes.c_void_p(out.data_ptr()), _stream(stream)))
        return out

    def embed_padded(self, ids, types, mask, batch: int, out=None, stream=None):
        """The padded bench loop from HOST numpy arrays: ids/types/mask int32 [n, seq]
        (types / mask may be None), batches of `batch` consecutive sentences with pipelined
        staging; returns the fp16 [n, 384] host array."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        n, seq = ids.shape
        types = None if types is None else np.ascontiguousarray(types, dtype=np.int32).reshape(n, seq)
        mask = None if mask is None else np.ascontiguousarray(mask, dtype=np.int32).reshape(n, seq)
        if out is None:
            out = np.zeros((n, HIDDEN), dtype=np.float16)
        if out.dtype != np.float16 or out.shape != (n, HIDDEN) or not out.flags.c_contiguous:
            raise ValueError("out must be a contiguous float16 [n, 384] host array")
        p = lambda a: None if a is None else a.ctypes.data_as(ctypes.c_void_p)
        _check(lib().bbh_embed_padded(self.handle, self.weights.handle, p(ids), p(types), p(mask), n, seq, int(batch),
                                      p(out), _stream(stream)))
        return out

    def free(self):
        if self.handle:
            lib().bbh_ws_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


# ---- WordPiece tokenizer (host only) --------------------------------------------------------
class Vocab:
    """BERT vocab.txt + WordPiece tokenization into the packed (ids, cu_seqlens) layout."""

    def __init__(self, path: str, lowercase: bool = True):
        self.handle = _P()
        _check(lib().bbh_vocab_load(path.encode(), 1 if lowercase else 0, ctypes.byref(self.handle)))

    def __len__(self):
        return lib().bbh_vocab_size(self.handle)

    def tokenize(self, texts, max_len: int = 128):
        """-> (ids int32 [total], cu_seqlens int32 [n+1]) for a list of str."""
        enc = [t.encode("utf-8") for t in texts]
        arr = (ctypes.c_char_p * max(len(enc), 1))(*enc)
        cu = np.zeros(len(enc) + 1, np.int32)
        total = ctypes.c_int64(0)
        cap = sum(min(len(e), 4 * max_len) for e in enc) + 2 * len(enc) + 16
        for _ in range(2):
            ids = np.empty(max(cap, 1), np.int32)
            rc = lib().bbh_tokenize(self.handle, ctypes.cast(arr, ctypes.c_void_p), len(enc), max_len,
                                    ids.ctypes.data_as(ctypes.c_void_p), cap, cu.ctypes.data_as(ctypes.c_void_p),
                                    ctypes.byref(total))
            if rc == BBH_OK:
                return ids[:total.value].copy(), cu
            if rc != -2:
                _check(rc)
            cap = total.value
        _check(rc)

    def free(self):
        if self.handle:
            lib().bbh_vocab_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


# ---- weight blob (host only) ---------------------------------------------------------------
def pack_weights(directory: str, layers: int, path: str) -> None:
    """<directory>/<HF key>.bin per-tensor files -> one checked blob file."""
    _check(lib().bbh_weights_pack(directory.encode(), layers, path.encode()))


def blob_check(path: str) -> int:
    """Validates a weight blob; returns its layer count (raises BBHError on corruption)."""
    n = ctypes.c_int(0)
    _check(lib().bbh_blob_check(path.encode(), ctypes.byref(n)))
    return n.value


# ---- host corpus planning ---------------------------------------------------------------
class CorpusPlan:
    """bbh_plan_batches result: order [n] (corpus indices, length-sorted), batch b =
    order[batch_first[b]:batch_first[b+1]], batch_rank [n_batches]."""

    def __init__(self, order, batch_first, batch_rank, n_batches):
        self.order, self.batch_first, self.batch_rank, self.n_batches = order, batch_first, batch_rank, n_batches

    def rank_order(self, rank: int) -> np.ndarray:
        """Corpus indices of `rank`'s sentences in plan order (its batches back to back)."""
        parts = [idx for _, idx in self.batches(rank)]
        return np.concatenate(parts) if parts else np.zeros(0, np.int32)

    def batches(self, rank=None):
        for b in range(self.n_batches):
            if rank is None or self.batch_rank[b] == rank:
                yield b, self.order[self.batch_first[b]:self.batch_first[b + 1]]


def plan_batches(lengths, max_batch: int, max_tokens: int, world: int = 1) -> CorpusPlan:
    """Length-sorted batches of at most max_batch sentences / max_tokens tokens, assigned to
    `world` ranks by longest-processing-time on their FLOPs (host only, no GPU needed)."""
    lengths = np.ascontiguousarray(lengths, dtype=np.int32)
    n = lengths.size
    order = np.empty(n, np.int32)
    first = np.empty(n + 1, np.int32)
    rank = np.empty(max(n, 1), np.int32)
    nb = ctypes.c_int(0)
    p = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    _check(lib().bbh_plan_batches(p(lengths), n, max_batch, max_tokens, world, p(order), p(first), p(rank),
                                  ctypes.byref(nb)))
    k = nb.value
    return CorpusPlan(order, first[:k + 1].copy(), rank[:k].copy(), k)


# ---- similarity evaluation (the step after the path) ---------------------------------------
def pair_similarity(emb, pairs, stream=None):
    """emb fp16 [n, 384], pairs int32 [m, 2] (CUDA tensors) -> fp32 [m] dot products."""
    if pairs.dtype != torch.int32 or pairs.dim() != 2 or pairs.shape[1] != 2:
        raise ValueError("pairs must be int32 [m, 2]")
    sims = torch.empty(pairs.shape[0], dtype=torch.float32, device=emb.device)
    _check(lib().bbh_pair_similarity(_f16(emb), emb.shape[0], _ptr(pairs), pairs.shape[0], _ptr(sims),
                                     _stream(stream)))
    return sims


def spearman(x, y) -> float:
    """Spearman rank correlation of two host sequences (average ranks for ties)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.ascontiguousarray(y, dtype=np.float32)
    if x.shape != y.shape:
        raise ValueError("x and y differ in length")
    rho = ctypes.c_double(0.0)
    _check(lib().bbh_spearman(x.ctypes.data_as(ctypes.c_void_p), y.ctypes.data_as(ctypes.c_void_p), x.size,
                              ctypes.byref(rho)))
    return rho.value


# ---- unit operators ---------------------------------------------------------------------
def set_gemm_pairs(mode: int) -> None:
    """Process-wide default GEMM tile mode for the unit operators and for workspaces created
    afterwards (Workspace.set_gemm_pairs sets one workspace's): 0 = one SM per 128-row tile,
    1 = SM pairs (256 x 192 where N allows, else 256 x 256), 2 (default) = SM pairs, 256 x 256
    first."""
    _check(lib().bbh_set_gemm_pairs(int(mode)))


def linear(A, W, bias=None, gelu=False, stream=None):
    """launch_matmul: A [M,K] @ W[N,K]^T (+bias) (+gelu) on the tcgen05 GEMM."""
    M, K = A.shape
    N = W.shape[0]
    C = torch.empty((M, N), dtype=torch.float16, device=A.device)
    _check(lib().bbh_linear(_f16(A), _f16(W), _f16(bias), _f16(C), M, N, K, 1 if gelu else 0, _stream(stream)))
    return C


def linear_residual_layernorm(A, W, bias, residual, gamma, beta, eps=1e-12, stream=None):
    M, K = A.shape
    C = torch.empty((M, HIDDEN), dtype=torch.float16, device=A.device)
    _check(lib().bbh_linear_residual_layernorm(_f16(A), _f16(W), _f16(bias), _f16(residual), _f16(gamma),
                                               _f16(beta), eps, _f16(C), M, K, _stream(stream)))
    return C


def layernorm(x, gamma, beta, eps=1e-12, residual=None, stream=None):
    M, D = x.shape
    y = torch.empty_like(x)
    _check(lib().bbh_layernorm(_f16(x), _f16(gamma), _f16(beta), _f16(y), M, D, eps, _f16(residual),
                               _stream(stream)))
    return y


def attention_varlen(qkv, cu_seqlens, max_len: int, keymask=None, stream=None):
    T = qkv.shape[0]
    ctx = torch.empty((T, HIDDEN), dtype=torch.float16, device=qkv.device)
    km = None
    if keymask is not None:
        if keymask.dtype != torch.uint8:
            raise TypeError("keymask must be uint8")
        km = _ptr(keymask)
    _check(lib().bbh_attention_varlen(_f16(qkv), _f16(ctx), _i32(cu_seqlens), km, cu_seqlens.numel() - 1, max_len,
                                      _stream(stream)))
    return ctx


def mean_pool_l2(hidden, cu_seqlens, tokmask=None, stream=None):
    B = cu_seqlens.numel() - 1
    emb = torch.empty((B, HIDDEN), dtype=torch.float16, device=hidden.device)
    tm = None
    if tokmask is not None:
        if tokmask.dtype != torch.uint8:
            raise TypeError("tokmask must be uint8")
        tm = _ptr(tokmask)
    _check(lib().bbh_mean_pool_l2(_f16(hidden), _i32(cu_seqlens), tm, B, _f16(emb), _stream(stream)))
    return emb
