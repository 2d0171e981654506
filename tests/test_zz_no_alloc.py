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


def test_static_entry_point_matches_workspace_entry_point():
    import bbh

    L = bbh.lib()
    gw = bbh.ModelWeights.from_numpy(om.make_weights(0), 6, 0)
    ws = bbh.Workspace(gw, 1024, 128, 64)
    dev = lambda a: torch.as_tensor(np.asarray(a), dtype=torch.int32).cuda()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for seed, n in ((31, 60), (32, 17)):  # two calls in a row, different shapes and tokens
        ids, types, cu = _packed(seed, n)
        assert int(cu[-1]) <= 1024
        d_ids, d_types, d_cu = dev(ids), dev(types), dev(cu)
        max_len = int(np.diff(cu).max())
        want = ws.embed_varlen(d_ids, d_types, d_cu, max_len)
        got = torch.full((n, 384), float("nan"), dtype=torch.float16, device="cuda")
        rc = L.bbh_embed_varlen_static(gw.handle, ctypes.c_void_p(d_ids.data_ptr()),
                                       ctypes.c_void_p(d_types.data_ptr()), ctypes.c_void_p(d_cu.data_ptr()), n,
                                       int(cu[-1]), max_len, ctypes.c_void_p(got.data_ptr()), stream)
        assert rc == 0, L.bbh_last_error()
        torch.cuda.synchronize()
        assert L.bbh_static_device_error() == 0
        g, w = got.float().cpu().numpy(), want.float().cpu().numpy()
        assert np.isfinite(g).all()
        cos = (g * w).sum(1) / (np.linalg.norm(g, axis=1) * np.linalg.norm(w, axis=1))
        assert cos.min() >= 0.9999
        assert np.abs(g - w).max() <= 2e-3


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
