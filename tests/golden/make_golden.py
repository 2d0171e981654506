"""Generate the golden fixtures in this folder (run: python tests/golden/make_golden.py).

The reference produces its goldens with scripts/dump_weights.py, which needs the
pretrained all-MiniLM-L6-v2 checkpoint and sentence-transformers (neither available
here). This script restates those dumps with the same arithmetic source the reference
uses -- transformers.BertModel on CPU fp32 -- over seeded random-init weights
(oracle.model.make_weights) and synthetic token ids:

  unit.npz   matmul (seed 0, shapes 4x16x8 and 128x384x384, x0.1), LayerNorm (seed 1,
             M=128 D=384), GELU (seed 2, n=128*1536, x1.5), softmax (seed 3, 128x128, x2)
             -- scripts/dump_weights.py:195-254. Inputs are regenerated from the seeds
             by the tests; only (a slice of) the outputs plus input checksums are stored.
  model.npz  expected_embedding / emb_out / attn0_out / layer0_out for one 9-token
             sentence padded to 128 (dump_weights.py:97-192), configs[0] batch
             embeddings, a lognormal varlen mini-corpus, perturbed-weight and 12-layer
             cases.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle import model as om  # noqa: E402


def unit_inputs():
    """Regenerate the unit-test inputs exactly as dump_weights.py:195-254 draws them."""
    out = {}
    rng = np.random.default_rng(0)
    for tag, M, N, K in (("small", 4, 16, 8), ("real", 128, 384, 384)):
        A = rng.standard_normal((M, K)).astype(np.float32) * 0.1
        B = rng.standard_normal((N, K)).astype(np.float32) * 0.1
        out[f"matmul_{tag}_A"] = A
        out[f"matmul_{tag}_B"] = B
    rng = np.random.default_rng(1)
    M, D = 128, 384
    out["ln_x"] = (rng.standard_normal((M, D)) * 1.0).astype(np.float16).astype(np.float32)
    out["ln_gamma"] = (rng.standard_normal((D,)) * 0.1 + 1.0).astype(np.float16).astype(np.float32)
    out["ln_beta"] = (rng.standard_normal((D,)) * 0.1).astype(np.float16).astype(np.float32)
    rng = np.random.default_rng(2)
    out["gelu_x"] = (rng.standard_normal(128 * 1536) * 1.5).astype(np.float16).astype(np.float32)
    rng = np.random.default_rng(3)
    out["softmax_x"] = (rng.standard_normal((128, 128)) * 2.0).astype(np.float16).astype(np.float32)
    return out


def bert_model(weights, layers):
    from transformers import BertConfig, BertModel

    cfg = BertConfig(vocab_size=om.VOCAB, hidden_size=om.HIDDEN, num_hidden_layers=layers,
                     num_attention_heads=om.HEADS, intermediate_size=om.FFN,
                     max_position_embeddings=om.MAX_POS, type_vocab_size=om.TYPES,
                     layer_norm_eps=om.EPS, hidden_act="gelu", attn_implementation="eager")
    bm = BertModel(cfg, add_pooling_layer=False).eval()
    bm.load_state_dict({k: torch.from_numpy(v.astype(np.float32)) for k, v in weights.items()}, strict=True)
    return bm


def bert_embed(bm, ids, types, mask):
    """dump_weights.py:108-120: last_hidden_state, masked mean, L2."""
    with torch.no_grad():
        h = bm(input_ids=torch.from_numpy(ids).long(), attention_mask=torch.from_numpy(mask).long(),
               token_type_ids=torch.from_numpy(types).long()).last_hidden_state
        m = torch.from_numpy(mask).unsqueeze(-1).float()
        pooled = (h * m).sum(dim=1) / m.sum(dim=1).clamp(min=1e-9)
        return (pooled / pooled.norm(dim=-1, keepdim=True).clamp(min=1e-12)).numpy()


def varlen_padded(cu, ids):
    lens = np.diff(cu)
    S = int(lens.max())
    pid = np.zeros((len(lens), S), np.int32)
    msk = np.zeros((len(lens), S), np.int32)
    for b, L in enumerate(lens):
        pid[b, :L] = ids[cu[b]:cu[b + 1]]
        msk[b, :L] = 1
    return pid, np.zeros_like(pid), msk


def main():
    u = unit_inputs()
    unit = {}
    for tag in ("small", "real"):
        A, B = u[f"matmul_{tag}_A"], u[f"matmul_{tag}_B"]
        C = A @ B.T
        unit[f"matmul_{tag}_C"] = C[:32].astype(np.float32)
    t = torch.from_numpy
    unit["ln_y"] = F.layer_norm(t(u["ln_x"]), (384,), t(u["ln_gamma"]), t(u["ln_beta"]), 1e-12).numpy()[:32]
    unit["gelu_y"] = F.gelu(t(u["gelu_x"])).numpy()[:8192]
    unit["softmax_y"] = F.softmax(t(u["softmax_x"]), dim=-1).numpy()[:32]
    for k, v in u.items():
        unit["sum_" + k] = np.float64(np.asarray(v, np.float64).sum())
    np.savez_compressed(os.path.join(HERE, "unit.npz"), **unit)

    mdl = {}
    w0 = om.make_weights(0)
    for k in ("embeddings.word_embeddings.weight", "encoder.layer.5.output.dense.weight"):
        mdl["wsum_" + k] = np.float64(w0[k].astype(np.float64).sum())
    bm = bert_model(w0, 6)

    # single sentence, 9 real tokens padded to 128 (dump_ref / dump_*_ref)
    ids, types, mask = om.padded_batch(1, 9, 128, seed=1)
    mdl["single_ids"], mdl["single_mask"] = ids, mask
    mdl["expected_embedding"] = bert_embed(bm, ids, types, mask)[0]
    with torch.no_grad():
        ii, tt, mm = (torch.from_numpy(a).long() for a in (ids, types, mask))
        emb = bm.embeddings(input_ids=ii, token_type_ids=tt)
        ext = (1.0 - mm[:, None, None, :].float()) * torch.finfo(torch.float32).min
        attn = bm.encoder.layer[0].attention(emb, attention_mask=ext)[0]
        lay = bm.encoder.layer[0](emb, attention_mask=ext)
        lay = lay[0] if isinstance(lay, tuple) else lay
    mdl["emb_out"] = emb[0, :16].numpy()
    mdl["attn0_out"] = attn[0, :16].numpy()
    mdl["layer0_out"] = lay[0, :16].numpy()

    # 64 x 9 tokens padded to 16
    ids, types, mask = om.padded_batch(64, 9, 16, seed=1)
    mdl["cfg0_embedding"] = bert_embed(bm, ids, types, mask)

    # lognormal varlen mini-corpus (configs[2] distribution), 24 sentences
    lens, rng = om.lognormal_lengths(24, seed=2)
    vids, vtypes, cu = om.packed_corpus(lens, rng)
    mdl["varlen_ids"], mdl["varlen_cu"] = vids, cu
    pid, pty, pmk = varlen_padded(cu, vids)
    mdl["varlen_embedding"] = bert_embed(bm, pid, pty, pmk)

    # perturbed weights (non-zero biases, LN affine), 8 sentences of configs[0]
    wp = om.make_weights(7, perturb=True)
    bmp = bert_model(wp, 6)
    ids, types, mask = om.padded_batch(8, 9, 16, seed=1)
    mdl["perturbed_embedding"] = bert_embed(bmp, ids, types, mask)

    # 12-layer variant, 2 sentences of 40 real tokens (configs[4] architecture)
    w12 = om.make_weights(4, layers=12)
    bm12 = bert_model(w12, 12)
    ids, types, mask = om.padded_batch(2, 40, 48, seed=4)
    mdl["l12_ids"], mdl["l12_mask"] = ids, mask
    mdl["l12_embedding"] = bert_embed(bm12, ids, types, mask)
    np.savez_compressed(os.path.join(HERE, "model.npz"), **mdl)
    print("wrote unit.npz, model.npz")


if __name__ == "__main__":
    main()
