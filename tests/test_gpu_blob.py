"""Weight blob on the GPU: weights loaded from one packed file give bit-identical
embeddings to the same weights loaded from the reference's per-tensor .bin folder, and a
corrupted blob is refused before anything is allocated."""
import time

import numpy as np
import pytest
import torch

from oracle import model as om

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")


def test_blob_loads_same_weights(tmp_path):
    import bbh
    import synthetic as sy

    w = om.make_weights(4, layers=6, perturb=True)
    om.save_weights(w, str(tmp_path / "weights"))
    blob = str(tmp_path / "w.bbhw")
    bbh.pack_weights(str(tmp_path / "weights"), 6, blob)
    bbh.ModelWeights.load_blob(blob, 0).free()  # context and allocator warm before timing
    t0 = time.perf_counter()
    a = bbh.ModelWeights.load(str(tmp_path / "weights"), 6, 0)
    t1 = time.perf_counter()
    b = bbh.ModelWeights.load_blob(blob, 0)
    t2 = time.perf_counter()
    print(f"load: per-tensor folder {1e3 * (t1 - t0):.1f} ms, blob {1e3 * (t2 - t1):.1f} ms")
    assert b.layers == 6
    rng = np.random.default_rng(4)
    lengths = rng.integers(5, 90, size=300).astype(np.int32)
    ids = sy.sentence_tokens(lengths, 4)
    offsets = np.zeros(301, np.int64)
    offsets[1:] = np.cumsum(lengths)
    plan = bbh.plan_batches(lengths, 128, 8192, 1)
    ea = bbh.Workspace(a, 8192, 128, 128).embed_corpus(ids, None, offsets, plan)
    eb = bbh.Workspace(b, 8192, 128, 128).embed_corpus(ids, None, offsets, plan)
    assert np.array_equal(ea.view(np.uint16), eb.view(np.uint16))
    raw = bytearray(open(blob, "rb").read())
    raw[len(raw) // 2] ^= 1
    bad = str(tmp_path / "bad.bbhw")
    open(bad, "wb").write(bytes(raw))
    with pytest.raises(bbh.BBHError) as e:
        bbh.ModelWeights.load_blob(bad, 0)
    assert e.value.code == -4
