"""Oracle: CPU fp32 restatement of the reference's sentence-embedding forward.

TEST INFRASTRUCTURE ONLY. Used by tests/, __graft_entry__.smoke() and the CPU-baseline
leg of bench.py as the checker; the product path never calls it.

What it restates (reference = tytrdev/bert-by-hand):
  * weights: per-tensor fp16 ``<HF state_dict key>.bin`` files, nn.Linear (out, in)
    row-major (scripts/dump_weights.py:69-94, src/model/weights.h:88-107).
  * embeddings: word[id] + pos[row % S] + type[tt], then LayerNorm eps 1e-12
    (src/kernels/embedding.cu:8-31, src/model/forward.cu:28-31).
  * encoder layer: fused QKV projection, scaled dot-product attention with key
    padding mask, output projection + residual + LayerNorm, intermediate dense +
    erf-GELU, output dense + residual + LayerNorm (src/model/encoder.cu:25-71).
    Masking follows the reference's golden generator: an additive finfo.min mask on
    padded keys (scripts/dump_weights.py:165-166).
  * pooling: (h * m).sum(1) / m.sum(1).clamp(1e-9), then x / ||x||.clamp(1e-12)
    (scripts/dump_weights.py:117-120; src/kernels/pooling.cu:8-32,
    src/kernels/normalize.cu:10-33).
The reference computes its goldens with transformers.BertModel (a third-party module
pinned at transformers 5.9.0 in the reference's uv.lock; 5.5.0 is installed here).
``tests/test_oracle_cpu.py`` pins this restatement against BertModel itself and against
the committed golden fixtures in tests/golden/.

Weights are seeded random init (no network, no pretrained checkpoint): matrices
N(0, 0.02), biases 0, LayerNorm gamma 1 / beta 0, word row 0 (pad id) zeroed, the same
distribution transformers' BertModel init uses. ``perturb=True`` additionally draws
non-zero biases and LayerNorm affine parameters so tests exercise those paths.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass

import numpy as np
import torch
import torch.nn.functional as F

VOCAB = 30522
HIDDEN = 384
HEADS = 12
HEAD_DIM = 32
FFN = 1536
MAX_POS = 512
TYPES = 2
EPS = 1e-12


def tensor_specs(layers: int = 6):
    """(HF state_dict key, shape) in BertModel state_dict order (101 tensors for L6).

    Same keys the reference loader reads (src/model/weights.h:58-71, 91-98).
    """
    specs = [
        ("embeddings.word_embeddings.weight", (VOCAB, HIDDEN)),
        ("embeddings.position_embeddings.weight", (MAX_POS, HIDDEN)),
        ("embeddings.token_type_embeddings.weight", (TYPES, HIDDEN)),
        ("embeddings.LayerNorm.weight", (HIDDEN,)),
        ("embeddings.LayerNorm.bias", (HIDDEN,)),
    ]
    for i in range(layers):
        p = f"encoder.layer.{i}."
        for part in ("query", "key", "value"):
            specs.append((p + f"attention.self.{part}.weight", (HIDDEN, HIDDEN)))
            specs.append((p + f"attention.self.{part}.bias", (HIDDEN,)))
        specs += [
            (p + "attention.output.dense.weight", (HIDDEN, HIDDEN)),
            (p + "attention.output.dense.bias", (HIDDEN,)),
            (p + "attention.output.LayerNorm.weight", (HIDDEN,)),
            (p + "attention.output.LayerNorm.bias", (HIDDEN,)),
            (p + "intermediate.dense.weight", (FFN, HIDDEN)),
            (p + "intermediate.dense.bias", (FFN,)),
            (p + "output.dense.weight", (HIDDEN, FFN)),
            (p + "output.dense.bias", (HIDDEN,)),
            (p + "output.LayerNorm.weight", (HIDDEN,)),
            (p + "output.LayerNorm.bias", (HIDDEN,)),
        ]
    return specs


def make_weights(seed: int = 0, layers: int = 6, perturb: bool = False) -> dict:
    """Seeded random-init fp16 weights, keyed by HF state_dict name."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape in tensor_specs(layers):
        if name.endswith("LayerNorm.weight"):
            a = np.ones(shape, np.float32)
            if perturb:
                a += rng.standard_normal(shape, dtype=np.float32) * 0.1
        elif name.endswith("bias"):
            a = np.zeros(shape, np.float32)
            if perturb:
                a = rng.standard_normal(shape, dtype=np.float32) * 0.05
        else:
            a = rng.standard_normal(shape, dtype=np.float32) * 0.02
            if name == "embeddings.word_embeddings.weight":
                a[0] = 0.0  # pad_token_id row, zeroed as BertModel's init does
        out[name] = a.astype(np.float16)
    return out


def save_weights(weights: dict, directory: str) -> None:
    """Write one ``<key>.bin`` fp16 file per tensor (scripts/dump_weights.py:75-82)."""
    os.makedirs(directory, exist_ok=True)
    for name, a in weights.items():
        np.ascontiguousarray(a, dtype=np.float16).tofile(os.path.join(directory, name + ".bin"))


def load_weights(directory: str, layers: int = 6) -> dict:
    out = {}
    for name, shape in tensor_specs(layers):
        a = np.fromfile(os.path.join(directory, name + ".bin"), dtype=np.float16)
        if a.size != int(np.prod(shape)):
            raise IOError(f"{name}: expected {np.prod(shape)} elements, got {a.size}")
        out[name] = a.reshape(shape)
    return out


@dataclass
class Oracle:
    """fp32 CPU forward over fp16-rounded weights (no weight-quantisation error)."""

    weights: dict
    layers: int = 6

    def __post_init__(self):
        self.t = {k: torch.from_numpy(v.astype(np.float32)) for k, v in self.weights.items()}

    # --- unit ops (each mirrors one reference launcher) -------------------------------
    @staticmethod
    def linear(x, w, b=None, gelu=False):
        """C = x @ w^T (+ b) (+ erf-GELU): src/kernels/matmul.cu:23-30, 164-186."""
        y = x @ w.T
        if b is not None:
            y = y + b
        return F.gelu(y) if gelu else y

    @staticmethod
    def layernorm(x, g, b, residual=None, eps=EPS):
        """LN(x [+ residual]): src/kernels/layernorm.cu:17-59."""
        if residual is not None:
            x = x + residual
        return F.layer_norm(x, (x.shape[-1],), g, b, eps)

    def _p(self, name):
        return self.t[name]

    def embeddings(self, ids, types, positions):
        """word + pos + type, LayerNorm: src/kernels/embedding.cu:20-30, forward.cu:28-31."""
        e = self._p("embeddings.word_embeddings.weight")[ids]
        e = e + self._p("embeddings.position_embeddings.weight")[positions]
        e = e + self._p("embeddings.token_type_embeddings.weight")[types]
        return self.layernorm(e, self._p("embeddings.LayerNorm.weight"), self._p("embeddings.LayerNorm.bias"))

    def layer(self, i, x, mask):
        """One post-LN encoder layer on padded [B, S, H] with key mask [B, S].

        src/model/encoder.cu:25-71; additive finfo.min key mask as in
        scripts/dump_weights.py:165-166.
        """
        p = f"encoder.layer.{i}."
        B, S, H = x.shape
        q = self.linear(x, self._p(p + "attention.self.query.weight"), self._p(p + "attention.self.query.bias"))
        k = self.linear(x, self._p(p + "attention.self.key.weight"), self._p(p + "attention.self.key.bias"))
        v = self.linear(x, self._p(p + "attention.self.value.weight"), self._p(p + "attention.self.value.bias"))

        def heads(t):
            return t.view(B, S, HEADS, HEAD_DIM).transpose(1, 2)

        s = heads(q) @ heads(k).transpose(-1, -2) / math.sqrt(HEAD_DIM)
        ext = (1.0 - mask[:, None, None, :].float()) * torch.finfo(torch.float32).min
        pr = torch.softmax(s + ext, dim=-1)
        ctx = (pr @ heads(v)).transpose(1, 2).reshape(B, S, H)
        a = self.layernorm(
            self.linear(ctx, self._p(p + "attention.output.dense.weight"), self._p(p + "attention.output.dense.bias")),
            self._p(p + "attention.output.LayerNorm.weight"), self._p(p + "attention.output.LayerNorm.bias"),
            residual=x,
        )
        h = self.linear(a, self._p(p + "intermediate.dense.weight"), self._p(p + "intermediate.dense.bias"), gelu=True)
        return self.layernorm(
            self.linear(h, self._p(p + "output.dense.weight"), self._p(p + "output.dense.bias")),
            self._p(p + "output.LayerNorm.weight"), self._p(p + "output.LayerNorm.bias"),
            residual=a,
        )

    @torch.inference_mode()
    def encode(self, ids, types, mask, dump_layers=False):
        """Padded forward: ids/types/mask int [B, S] -> hidden [B, S, 384] (forward.cu:20-42).

        Positions are row % S (embedding.cu:22). With dump_layers, also returns the
        hidden state after the embedding LN and after every layer.
        """
        ids = torch.as_tensor(np.asarray(ids), dtype=torch.long)
        types = torch.as_tensor(np.asarray(types), dtype=torch.long)
        mask = torch.as_tensor(np.asarray(mask), dtype=torch.long)
        B, S = ids.shape
        pos = torch.arange(S).expand(B, S)
        x = self.embeddings(ids, types, pos)
        dumps = [x.clone()] if dump_layers else None
        for i in range(self.layers):
            x = self.layer(i, x, mask)
            if dump_layers:
                dumps.append(x.clone())
        return (x, dumps) if dump_layers else x

    @staticmethod
    def pool_l2(hidden, mask):
        """Masked mean + L2 normalise (scripts/dump_weights.py:117-120)."""
        m = torch.as_tensor(np.asarray(mask)).unsqueeze(-1).float()
        pooled = (hidden * m).sum(dim=1) / m.sum(dim=1).clamp(min=1e-9)
        return pooled / pooled.norm(dim=-1, keepdim=True).clamp(min=1e-12)

    @torch.inference_mode()
    def embed(self, ids, types, mask):
        """bert_embed (forward.cu:44-53): [B, S] ids -> [B, 384] fp32 unit embeddings."""
        return self.pool_l2(self.encode(ids, types, mask), mask)

    @torch.inference_mode()
    def embed_varlen(self, ids, types, cu_seqlens, dump_layers=False):
        """Packed form: ids/types [T], cu_seqlens [B+1] -> [B, 384].

        Each sentence is padded to the batch maximum with a key mask, which is exactly
        the padded forward restricted to real tokens (sentences are independent).
        With dump_layers also returns per-layer hidden states packed as [T, 384].
        """
        ids = np.asarray(ids)
        types = np.asarray(types)
        cu = np.asarray(cu_seqlens)
        B = len(cu) - 1
        lens = np.diff(cu)
        S = int(lens.max()) if B else 0
        pid = np.zeros((B, S), np.int64)
        pty = np.zeros((B, S), np.int64)
        msk = np.zeros((B, S), np.int64)
        for b in range(B):
            L = lens[b]
            pid[b, :L] = ids[cu[b]:cu[b + 1]]
            pty[b, :L] = types[cu[b]:cu[b + 1]]
            msk[b, :L] = 1
        if dump_layers:
            x, dumps = self.encode(pid, pty, msk, dump_layers=True)
        else:
            x = self.encode(pid, pty, msk)
        emb = self.pool_l2(x, msk)
        if not dump_layers:
            return emb
        sel = torch.from_numpy(msk.reshape(-1).astype(bool))
        packed = [d.reshape(B * S, HIDDEN)[sel] for d in dumps]
        return emb, packed


def gather_indices(ids, types, mask=None, cu_seqlens=None) -> np.ndarray:
    """(word id, position id, type id, mask) per token as the reference's embedding and
    pooling kernels index them: padded [B, S] inputs use position = row % S
    (src/kernels/embedding.cu:20-25) and pool where mask != 0 (src/kernels/pooling.cu:23-28);
    a packed sentence is the same sentence padded on its own, so its positions restart at 0
    and every token is real. Returns int32 [T, 4] in the input's token order."""
    ids = np.asarray(ids)
    types = np.zeros_like(ids) if types is None else np.asarray(types)
    if cu_seqlens is not None:
        cu = np.asarray(cu_seqlens, np.int64)
        pos = np.concatenate([np.arange(cu[b + 1] - cu[b]) for b in range(len(cu) - 1)]) if len(cu) > 1 else []
        m = np.ones(ids.size, np.int64)
        return np.stack([ids.reshape(-1), np.asarray(pos, np.int64), types.reshape(-1), m], 1).astype(np.int32)
    B, S = ids.shape
    m = np.ones((B, S), np.int64) if mask is None else (np.asarray(mask) != 0).astype(np.int64)
    pos = np.broadcast_to(np.arange(S), (B, S))
    return np.stack([ids.reshape(-1), pos.reshape(-1), types.reshape(-1), m.reshape(-1)], 1).astype(np.int32)


# --- synthetic inputs (stand-ins for the reference's tokenised STS sentences) ----------

def sentence_ids(rng, length: int) -> np.ndarray:
    """[CLS]=101, interior ids uniform in [1000, 30521], [SEP]=102."""
    ids = np.empty(length, np.int32)
    ids[0] = 101
    ids[-1] = 102
    if length > 2:
        ids[1:-1] = rng.integers(1000, 30522, size=length - 2)
    return ids


def padded_batch(batch: int, real: int, seq: int, seed: int = 1):
    """configs[0]/[1]: `batch` sentences of `real` tokens padded with id 0 to `seq`."""
    rng = np.random.default_rng(seed)
    ids = np.zeros((batch, seq), np.int32)
    mask = np.zeros((batch, seq), np.int32)
    for b in range(batch):
        ids[b, :real] = sentence_ids(rng, real)
        mask[b, :real] = 1
    return ids, np.zeros_like(ids), mask


def lognormal_lengths(n: int, seed: int = 2, lo: int = 5, hi: int = 64):
    """L = clip(round(lognormal(ln 12, 0.555)), 5, 64) (median 12, mean ~14)."""
    rng = np.random.default_rng(seed)
    return np.clip(np.round(rng.lognormal(math.log(12.0), 0.555, size=n)), lo, hi).astype(np.int32), rng


def uniform_lengths(n: int, seed: int = 3, lo: int = 8, hi: int = 128):
    """L ~ U[lo, hi] inclusive."""
    rng = np.random.default_rng(seed)
    return rng.integers(lo, hi + 1, size=n).astype(np.int32), rng


def packed_corpus(lengths: np.ndarray, rng):
    """Packed ids/types [T] and cu_seqlens [B+1] for the given sentence lengths."""
    cu = np.zeros(len(lengths) + 1, np.int32)
    cu[1:] = np.cumsum(lengths)
    ids = np.concatenate([sentence_ids(rng, int(L)) for L in lengths]) if len(lengths) else np.zeros(0, np.int32)
    return ids.astype(np.int32), np.zeros_like(ids, dtype=np.int32), cu
