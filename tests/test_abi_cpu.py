"""The C-ABI library loads, exports every symbol include/bbh.h declares, and keeps the
reference's tensor catalogue -- all without a GPU (no compute calls)."""
import ctypes
import os
import re
import subprocess

import pytest

from oracle import model as om

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "bbh.h")).read()
    return sorted(set(re.findall(r"BBH_API\s+[\w\s\*]+?\b(bbh_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    import bbh

    L = bbh.lib()
    decl = declared_symbols()
    assert len(decl) >= 20
    for name in decl:
        assert hasattr(L, name), name
    assert sorted(bbh.exported_symbols()) == decl
    out = subprocess.run(["nm", "-D", "--defined-only", bbh.LIB_PATH], capture_output=True, text=True).stdout
    exported = sorted(set(re.findall(r" T (bbh_\w+)", out)))
    assert exported == decl


def test_tensor_catalogue_matches_reference_keys():
    import bbh

    for layers in (6, 12):
        assert bbh.tensor_names(layers) == [n for n, _ in om.tensor_specs(layers)]
        L = bbh.lib()
        for i, (_, shape) in enumerate(om.tensor_specs(layers)):
            assert L.bbh_tensor_numel(layers, i) == int(__import__("numpy").prod(shape))
    assert bbh.lib().bbh_num_tensors(6) == 101
    assert bbh.lib().bbh_num_tensors(7) == 0
    assert bbh.lib().bbh_tensor_name(6, 101) is None


def test_argument_errors_need_no_gpu(tmp_path):
    import bbh

    L = bbh.lib()
    h = ctypes.c_void_p()
    assert L.bbh_weights_load(b"/nonexistent", 6, 0, ctypes.byref(h)) == -4  # BBH_ERR_IO
    assert b"cannot open" in L.bbh_last_error()
    assert L.bbh_weights_load(None, 6, 0, ctypes.byref(h)) == -1
    assert L.bbh_weights_load(str(tmp_path).encode(), 5, 0, ctypes.byref(h)) == -1
    assert L.bbh_ws_create(None, 16, 1, 16, ctypes.byref(h)) == -1
    assert L.bbh_embed(None, None, None, None, None, None, 1, 16, None) == -1


def test_short_weight_file_is_rejected(tmp_path):
    import bbh

    w = om.make_weights(0)
    om.save_weights(w, str(tmp_path))
    p = tmp_path / "encoder.layer.3.output.dense.bias.bin"
    p.write_bytes(p.read_bytes()[:100])
    h = ctypes.c_void_p()
    assert bbh.lib().bbh_weights_load(str(tmp_path).encode(), 6, 0, ctypes.byref(h)) == -4
    assert b"expected 384 elements" in bbh.lib().bbh_last_error()


def test_product_path_does_not_import_oracle():
    pkg = os.path.join(ROOT, "bert-by-hand_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h", ".hpp", ".cpp")):
                text = open(os.path.join(dirpath, f)).read()
                assert "oracle" not in text.replace("Oracle", ""), f
