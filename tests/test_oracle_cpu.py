"""The CPU oracle, pinned against the golden fixtures and transformers.BertModel.

The fixtures come from tests/golden/make_golden.py, which restates the reference's
golden dumps (scripts/dump_weights.py:97-254) with BertModel on CPU fp32.
"""
import numpy as np
import pytest
import torch

from oracle import model as om
from tests.golden.make_golden import unit_inputs


def cos_rows(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return (a * b).sum(-1) / (np.linalg.norm(a, axis=-1) * np.linalg.norm(b, axis=-1) + 1e-30)


@pytest.fixture(scope="module")
def oracle6():
    return om.Oracle(om.make_weights(0))


def test_unit_inputs_regenerate_exactly(golden_unit):
    """The seeded unit inputs (dump_weights.py:195-254) regenerate bit-for-bit."""
    for k, v in unit_inputs().items():
        assert float(np.asarray(v, np.float64).sum()) == float(golden_unit["sum_" + k]), k


def test_unit_ops_match_golden(golden_unit):
    u = unit_inputs()
    t = torch.from_numpy
    for tag in ("small", "real"):
        C = om.Oracle.linear(t(u[f"matmul_{tag}_A"]), t(u[f"matmul_{tag}_B"])).numpy()
        np.testing.assert_allclose(C[:32], golden_unit[f"matmul_{tag}_C"], rtol=1e-5, atol=1e-6)
    y = om.Oracle.layernorm(t(u["ln_x"]), t(u["ln_gamma"]), t(u["ln_beta"])).numpy()
    np.testing.assert_allclose(y[:32], golden_unit["ln_y"], rtol=1e-5, atol=1e-5)
    g = om.Oracle.linear(t(u["gelu_x"][:, None]), torch.ones(1, 1), gelu=True).numpy()[:, 0]
    np.testing.assert_allclose(g[:8192], golden_unit["gelu_y"], rtol=1e-6, atol=1e-6)
    s = torch.softmax(t(u["softmax_x"]), -1).numpy()
    np.testing.assert_allclose(s[:32], golden_unit["softmax_y"], rtol=1e-6, atol=1e-7)


def test_weights_regenerate_exactly(golden_model):
    w = om.make_weights(0)
    for k in ("embeddings.word_embeddings.weight", "encoder.layer.5.output.dense.weight"):
        assert float(w[k].astype(np.float64).sum()) == float(golden_model["wsum_" + k])
    assert np.all(w["embeddings.word_embeddings.weight"][0] == 0)


def test_single_sentence_matches_golden(oracle6, golden_model):
    ids, mask = golden_model["single_ids"], golden_model["single_mask"]
    types = np.zeros_like(ids)
    emb = oracle6.embed(ids, types, mask).numpy()[0]
    assert cos_rows(emb, golden_model["expected_embedding"]) > 0.999999
    x, dumps = oracle6.encode(ids, types, mask, dump_layers=True)
    np.testing.assert_allclose(dumps[0][0, :16].numpy(), golden_model["emb_out"], atol=2e-5)
    np.testing.assert_allclose(dumps[1][0, :16].numpy(), golden_model["layer0_out"], atol=5e-5)


def test_padding_invariance(oracle6, golden_model):
    """Same 9 real tokens padded to 16 or to 128 give the same embedding (bench.cu:66-84)."""
    ids, mask = golden_model["single_ids"], golden_model["single_mask"]
    e128 = oracle6.embed(ids, np.zeros_like(ids), mask).numpy()
    e16 = oracle6.embed(ids[:, :16], np.zeros_like(ids[:, :16]), mask[:, :16]).numpy()
    assert cos_rows(e128, e16).min() > 0.999999


def test_cfg0_batch_matches_golden(oracle6, golden_model):
    ids, types, mask = om.padded_batch(64, 9, 16, seed=1)
    emb = oracle6.embed(ids, types, mask).numpy()
    assert cos_rows(emb, golden_model["cfg0_embedding"]).min() > 0.999999


def test_varlen_matches_golden(oracle6, golden_model):
    ids, cu = golden_model["varlen_ids"], golden_model["varlen_cu"]
    emb = oracle6.embed_varlen(ids, np.zeros_like(ids), cu).numpy()
    assert cos_rows(emb, golden_model["varlen_embedding"]).min() > 0.999999


def test_perturbed_and_l12_match_golden(golden_model):
    o = om.Oracle(om.make_weights(7, perturb=True))
    ids, types, mask = om.padded_batch(8, 9, 16, seed=1)
    assert cos_rows(o.embed(ids, types, mask).numpy(), golden_model["perturbed_embedding"]).min() > 0.999999
    o12 = om.Oracle(om.make_weights(4, layers=12), layers=12)
    ids, mask = golden_model["l12_ids"], golden_model["l12_mask"]
    e = o12.embed(ids, np.zeros_like(ids), mask).numpy()
    assert cos_rows(e, golden_model["l12_embedding"]).min() > 0.999999


def test_oracle_equals_bertmodel_directly():
    """Pin against the reference's arithmetic source (transformers.BertModel)."""
    pytest.importorskip("transformers")
    from tests.golden.make_golden import bert_model

    w = om.make_weights(11, perturb=True)
    bm = bert_model(w, 6)
    ids, types, mask = om.padded_batch(3, 20, 24, seed=5)
    mask[1, 15:] = 0
    with torch.no_grad():
        ref = bm(input_ids=torch.from_numpy(ids).long(), attention_mask=torch.from_numpy(mask).long(),
                 token_type_ids=torch.from_numpy(types).long()).last_hidden_state
    got = om.Oracle(w).encode(ids, types, mask)
    assert (ref - got).abs().max().item() < 1e-4


def test_varlen_equals_padded_on_real_tokens(oracle6):
    lens, rng = om.lognormal_lengths(6, seed=9)
    ids, types, cu = om.packed_corpus(lens, rng)
    emb, dumps = oracle6.embed_varlen(ids, types, cu, dump_layers=True)
    assert len(dumps) == 7 and dumps[-1].shape == (int(cu[-1]), 384)
    # one sentence at a time gives the same answer
    for b in range(len(lens)):
        one = oracle6.embed_varlen(ids[cu[b]:cu[b + 1]], types[cu[b]:cu[b + 1]], np.array([0, lens[b]]))
        assert cos_rows(one.numpy(), emb[b:b + 1].numpy()).min() > 0.999999


def test_weight_files_roundtrip(tmp_path):
    w = om.make_weights(3)
    om.save_weights(w, str(tmp_path))
    back = om.load_weights(str(tmp_path))
    for k in w:
        assert np.array_equal(w[k], back[k])
