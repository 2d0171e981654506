"""Seeded synthetic inputs for benchmarking the engine (no network, no checkpoints).

* weights: MiniLM/BERT random init -- matrices N(0, 0.02), biases 0, LayerNorm gamma 1 /
  beta 0, word row 0 zeroed -- as fp16 arrays keyed by HF state_dict name (the names the
  reference's weight files carry, scripts/dump_weights.py:75-82).
* sentences: [CLS]=101, interior ids uniform in [1000, 30521], [SEP]=102; lengths drawn
  per workload (uniform for the throughput sweep, log-normal for the STS-like corpus that
  stands in for the reference's 2000 STS sentences, bench/corpus.cu).
* batching: sort by length, cut into fixed-size batches, pack each with cu_seqlens
  (the reference's dynamic batching, bench/corpus.cu:80-118, without the padding).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

import bbh


def random_weights(seed: int = 0, layers: int = 6) -> dict:
    rng = np.random.default_rng(seed)
    out = {}
    for name in bbh.tensor_names(layers):
        n = bbh.lib().bbh_tensor_numel(layers, bbh.tensor_names(layers).index(name))
        if name.endswith("LayerNorm.weight"):
            a = np.ones(n, np.float16)
        elif name.endswith("bias"):
            a = np.zeros(n, np.float16)
        else:
            a = (rng.standard_normal(n, dtype=np.float32) * 0.02).astype(np.float16)
            if name == "embeddings.word_embeddings.weight":
                a[:384] = 0
        out[name] = a
    return out


def lengths_uniform(n: int, lo: int, hi: int, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).integers(lo, hi + 1, size=n).astype(np.int32)


def lengths_lognormal(n: int, seed: int, lo: int = 5, hi: int = 64) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return np.clip(np.round(rng.lognormal(math.log(12.0), 0.555, size=n)), lo, hi).astype(np.int32)


def sentence_tokens(lengths: np.ndarray, seed: int) -> np.ndarray:
    """Packed ids for sentences of the given lengths (vectorised)."""
    rng = np.random.default_rng(seed + 7919)
    T = int(lengths.sum())
    ids = rng.integers(1000, 30522, size=T).astype(np.int32)
    ends = np.cumsum(lengths)
    starts = ends - lengths
    ids[starts] = 101
    ids[ends - 1] = 102
    return ids


@dataclass
class Batch:
    first: int          # index of the batch's first sentence in sorted order
    count: int          # sentences in the batch
    tok_start: int      # offset of its first token in the packed token array
    tokens: int         # total tokens
    max_len: int
    cu: np.ndarray      # [count + 1] int32, relative to tok_start


@dataclass
class Corpus:
    order: np.ndarray   # sorted position -> original sentence index
    ids: np.ndarray     # packed ids in sorted order
    types: np.ndarray
    batches: list


def bucketed_corpus(lengths: np.ndarray, batch: int, seed: int) -> Corpus:
    """Length-sorted, batched, packed corpus."""
    order = np.argsort(lengths, kind="stable")
    sl = lengths[order]
    ids = sentence_tokens(sl, seed)
    ends = np.cumsum(sl)
    batches = []
    for s in range(0, len(sl), batch):
        e = min(s + batch, len(sl))
        tok0 = int(ends[s - 1]) if s else 0
        cu = np.zeros(e - s + 1, np.int32)
        cu[1:] = np.cumsum(sl[s:e])
        batches.append(Batch(s, e - s, tok0, int(cu[-1]), int(sl[s:e].max()), cu))
    return Corpus(order, ids, np.zeros_like(ids), batches)


def batch_flops(lengths: np.ndarray, layers: int = 6) -> float:
    """Algorithmic FLOPs: 3,538,944 GEMM FLOPs per token per layer + 4*L^2*384 attention."""
    L = lengths.astype(np.float64)
    return float(layers * (3538944.0 * L.sum() + 4.0 * 384.0 * (L * L).sum()))
