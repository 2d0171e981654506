"""The no-allocation entry point, bbh_embed_varlen_static, called through the C ABI.

It exists for callers that cannot call cudaMalloc -- hosts whose pool allocator owns all
device memory, or latency-critical code that cannot take an allocation's implicit
synchronisation -- and keeps its scratch in a fixed device array inside libbbh.so. Its
output must equal the regular workspace entry point's (bbh_embed_varlen) on two calls in a
row with different inputs, so nothing left in the shared array from the first call leaks
into the second. This file is collected last on purpose.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import model as om

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")


def _packed(seed, n):
    lens, rng = om.lognormal_lengths(n, seed=seed)
    return om.packed_corpus(lens, rng)


def _call_static(L, gw, d_ids, d_types, d_cu, n, total, max_len, out, stream):
    return L.bbh_embed_varlen_static(gw.handle, ctypes.c_void_p(d_ids.data_ptr()),
                                     ctypes.c_void_p(d_types.data_ptr()) if d_types is not None else None,
                                     ctypes.c_void_p(d_cu.data_ptr()), n, total, max_len,
                                     ctypes.c_void_p(out.data_ptr()), stream)


def _long_batch(seed):
    """Sentences of 129-512 tokens (the long-sentence attention kernel) next to short ones,
    1,024 tokens in all (the static array's limit)."""
    rng = np.random.default_rng(seed)
    lens = np.array([300, 200, 129, 150, 17, 64, 100, 1, 63], np.int64)
    lens[-1] = 1024 - int(lens[:-1].sum())
    ids = np.concatenate([om.sentence_ids(rng, int(x)) for x in lens]).astype(np.int32)
    cu = np.zeros(lens.size + 1, np.int32)
    cu[1:] = np.cumsum(lens)
    return ids, (rng.random(ids.size) < 0.2).astype(np.int32), cu


def test_static_entry_point_matches_workspace_entry_point():
    """Two calls in a row with different inputs (a short-sentence batch, then one with
    sentences of 129-512 tokens), each bit for bit equal to bbh_embed_varlen: the same
    kernels on the same inputs, so any difference would be state left in the shared array."""
    import bbh

    L = bbh.lib()
    gw = bbh.ModelWeights.from_numpy(om.make_weights(0), 6, 0)
    ws = bbh.Workspace(gw, 1024, 128, 512)
    dev = lambda a: torch.as_tensor(np.asarray(a), dtype=torch.int32).cuda()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    cases = [_packed(31, 60), _long_batch(32), _packed(33, 17)]
    for ids, types, cu in cases:
        n = len(cu) - 1
        assert int(cu[-1]) <= 1024
        d_ids, d_types, d_cu = dev(ids), dev(types), dev(cu)
        max_len = int(np.diff(cu).max())
        want = ws.embed_varlen(d_ids, d_types, d_cu, max_len)
        got = torch.full((n, 384), float("nan"), dtype=torch.float16, device="cuda")
        rc = _call_static(L, gw, d_ids, d_types, d_cu, n, int(cu[-1]), max_len, got, stream)
        assert rc == 0, L.bbh_last_error()
        torch.cuda.synchronize()
        assert L.bbh_static_device_error() == 0
        assert ws.device_error() == 0
        assert torch.isfinite(got.float()).all()
        assert torch.equal(got, want)


def test_static_entry_point_reports_device_errors():
    """A token id outside the vocabulary is flagged in the static path's own error word,
    and the next good call starts from a cleared word."""
    import bbh

    L = bbh.lib()
    gw = bbh.ModelWeights.from_numpy(om.make_weights(0), 6, 0)
    ids = torch.full((20,), 1000, dtype=torch.int32, device="cuda")
    ids[5] = 40000
    cu = torch.tensor([0, 8, 20], dtype=torch.int32, device="cuda")
    out = torch.empty((2, 384), dtype=torch.float16, device="cuda")
    assert _call_static(L, gw, ids, None, cu, 2, 20, 12, out, None) == 0
    torch.cuda.synchronize()
    assert L.bbh_static_device_error() == 2
    ids[5] = 1000
    assert _call_static(L, gw, ids, None, cu, 2, 20, 12, out, None) == 0
    torch.cuda.synchronize()
    assert L.bbh_static_device_error() == 0


def test_static_entry_point_rejects_oversized_requests():
    import bbh

    L = bbh.lib()
    gw = bbh.ModelWeights.from_numpy(om.make_weights(0), 6, 0)
    ids = torch.full((2000,), 1000, dtype=torch.int32, device="cuda")
    cu = torch.tensor([0, 1000, 2000], dtype=torch.int32, device="cuda")
    out = torch.empty((2, 384), dtype=torch.float16, device="cuda")
    rc = L.bbh_embed_varlen_static(gw.handle, ctypes.c_void_p(ids.data_ptr()), None, ctypes.c_void_p(cu.data_ptr()),
                                   2, 2000, 1000, ctypes.c_void_p(out.data_ptr()), None)
    assert rc == -2
    assert b"static scratch" in L.bbh_last_error()
    # a sentence longer than the 512-entry position table, inside the token limit
    small = torch.full((600,), 1000, dtype=torch.int32, device="cuda")
    cu1 = torch.tensor([0, 600], dtype=torch.int32, device="cuda")
    rc = L.bbh_embed_varlen_static(gw.handle, ctypes.c_void_p(small.data_ptr()), None,
                                   ctypes.c_void_p(cu1.data_ptr()), 1, 600, 600, ctypes.c_void_p(out.data_ptr()), None)
    assert rc == -2
    assert b"512" in L.bbh_last_error()
