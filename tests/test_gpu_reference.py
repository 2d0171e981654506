"""Second oracle: the reference's own CUDA implementation (built from its unmodified
sources into oracle/_ref/libbbh_ref.so by oracle/Makefile) run on the same B200, same
weight files and same inputs; plus the C++ drop-in example through include/bert_by_hand.hpp.

The reference accumulates its GEMMs and attention in fp16 (src/kernels/matmul.cu:110,
attention.cu:32), so it is held to its own gate (cosine >= 0.999, tests/test_embed.cu:34)
against our output, with max-abs reported."""
import ctypes
import os
import subprocess

import numpy as np
import pytest
import torch

from oracle import model as om

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libbbh_ref.so")
EXAMPLE = os.path.join(ROOT, "bert-by-hand_b200", "_build", "bert_embed_main")


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")


@pytest.fixture(scope="module")
def weights_root(tmp_path_factory):
    root = tmp_path_factory.mktemp("refw")
    om.save_weights(om.make_weights(0), str(root / "weights"))
    return str(root)


def cos_rows(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return (a * b).sum(-1) / (np.linalg.norm(a, axis=-1) * np.linalg.norm(b, axis=-1) + 1e-30)


def ours(weights_root, ids, types, mask):
    import bbh

    gw = bbh.ModelWeights.load(os.path.join(weights_root, "weights"), 6, 0)
    B, S = ids.shape
    ws = bbh.Workspace(gw, B * S, B, S)
    d = lambda a: torch.as_tensor(a, dtype=torch.int32).cuda()
    e = ws.embed(d(ids), d(types), d(mask))
    torch.cuda.synchronize()
    return e.float().cpu().numpy()


def ref_cuda(weights_root, ids, types, mask):
    if not os.path.exists(REF_LIB):
        pytest.skip("oracle/_ref/libbbh_ref.so not built (needs the reference sources at build time)")
    L = ctypes.CDLL(REF_LIB)
    B, S = ids.shape
    out = np.zeros((B, 384), np.float16)
    ms = ctypes.c_float(0)
    i32 = lambda a: np.ascontiguousarray(a, np.int32).ctypes.data_as(ctypes.c_void_p)
    keep = [np.ascontiguousarray(a, np.int32) for a in (ids, types, mask)]
    rc = L.ref_embed(weights_root.encode(), *(a.ctypes.data_as(ctypes.c_void_p) for a in keep),
                     out.ctypes.data_as(ctypes.c_void_p), B, S, 0, ctypes.byref(ms))
    assert rc == 0
    return out.astype(np.float32)


@pytest.mark.parametrize("batch,real,seq", [(64, 9, 16), (64, 9, 128), (16, 40, 64), (8, 128, 128)])
def test_matches_reference_cuda(weights_root, batch, real, seq):
    ids, types, mask = om.padded_batch(batch, real, seq, seed=1)
    r = ref_cuda(weights_root, ids, types, mask)
    o = ours(weights_root, ids, types, mask)
    t = om.Oracle(om.load_weights(os.path.join(weights_root, "weights"))).embed(ids, types, mask).numpy()
    c_ref = cos_rows(o, r)
    print(f"B{batch} S{seq}: cos(ours, ref-cuda) min {c_ref.min():.6f}, max-abs {np.abs(o - r).max():.3e}; "
          f"cos(ref-cuda, torch) min {cos_rows(r, t).min():.6f}; cos(ours, torch) min {cos_rows(o, t).min():.6f}")
    assert c_ref.min() >= 0.999
    assert cos_rows(o, t).min() >= 0.9999


def test_corpus_loop_matches_reference_cuda(weights_root):
    """The reference's dynamic-length corpus loop (bench/corpus.cu:80-128: length-sorted
    batches of 64, each padded to its longest rounded to 16) over a configs[2]-style corpus,
    against bbh_embed_corpus on the same sentences (packed, token-bounded batches)."""
    import bbh

    if not os.path.exists(REF_LIB):
        pytest.skip("oracle/_ref/libbbh_ref.so not built")
    lens, rng = om.lognormal_lengths(700, seed=2)
    ids, types, cu = om.packed_corpus(lens, rng)
    L = ctypes.CDLL(REF_LIB)
    ref = np.zeros((lens.size, 384), np.float16)
    p = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    ids32, cu32 = np.ascontiguousarray(ids, np.int32), np.ascontiguousarray(cu, np.int32)
    assert L.ref_corpus(weights_root.encode(), p(ids32), p(cu32), int(lens.size), 64, 0, None, p(ref)) == 0
    gw = bbh.ModelWeights.load(os.path.join(weights_root, "weights"), 6, 0)
    ws = bbh.Workspace(gw, 64 * 64, 64, 64)
    plan = bbh.plan_batches(lens, 64, 64 * 64, 1)
    ours_emb = ws.embed_corpus(ids, types, cu.astype(np.int64), plan)
    c = cos_rows(ours_emb.astype(np.float32), ref.astype(np.float32))
    print(f"corpus loop: cos(ours, ref-cuda) min {c.min():.6f}")
    assert c.min() >= 0.999


def test_cpp_dropin_example(weights_root, tmp_path):
    """bert_embed through include/bert_by_hand.hpp equals the C-ABI result bit for bit."""
    if not os.path.exists(EXAMPLE):
        pytest.skip("example not built")
    ids, types, mask = om.padded_batch(32, 12, 32, seed=3)
    for name, a in (("ids", ids), ("types", types), ("mask", mask)):
        np.ascontiguousarray(a, np.int32).tofile(tmp_path / f"{name}.bin")
    out = tmp_path / "emb.bin"
    r = subprocess.run([EXAMPLE, os.path.join(weights_root, "weights"), str(tmp_path / "ids.bin"),
                        str(tmp_path / "types.bin"), str(tmp_path / "mask.bin"), "32", "32", str(out)],
                       capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    got = np.fromfile(out, np.float16).reshape(32, 384).astype(np.float32)
    want = ours(weights_root, ids, types, mask)
    assert np.array_equal(got, want)
