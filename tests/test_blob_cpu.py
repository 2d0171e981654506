"""Weight blob (host only): per-tensor .bin files (the reference's weights/ layout) packed
into one checked file; the checker accepts the result, reports its layer count, and
rejects truncation, corrupted data, a wrong magic and a missing tensor file."""
import os
import struct

import numpy as np
import pytest

from oracle import model as om


@pytest.fixture(scope="module")
def packed(tmp_path_factory):
    import bbh

    d = tmp_path_factory.mktemp("w")
    w = om.make_weights(3, layers=6, perturb=True)
    om.save_weights(w, str(d / "weights"))
    blob = str(d / "minilm.bbhw")
    bbh.pack_weights(str(d / "weights"), 6, blob)
    return bbh, w, blob, d


def test_pack_and_check(packed):
    bbh, w, blob, d = packed
    assert bbh.blob_check(blob) == 6
    raw = open(blob, "rb").read()
    assert raw[:4] == b"BBHW"
    version, layers, count, data_off, data_bytes = struct.unpack_from("<IIIQQ", raw, 4)
    assert (version, layers, count) == (1, 6, bbh.lib().bbh_num_tensors(6)) and data_off % 4096 == 0
    # walk the table: every tensor's bytes equal its .bin file
    at = 40
    for i in range(count):
        (n,) = struct.unpack_from("<I", raw, at)
        name = raw[at + 4:at + 4 + n].decode()
        numel, off = struct.unpack_from("<QQ", raw, at + 4 + n)
        at += 4 + n + 16
        assert name == bbh.tensor_names(6)[i] and off % 256 == 0
        got = np.frombuffer(raw, np.float16, count=numel, offset=data_off + off)
        assert np.array_equal(got.view(np.uint16), np.ascontiguousarray(w[name], np.float16).view(np.uint16).ravel())


def test_check_rejects_damage(packed):
    bbh, w, blob, d = packed
    raw = bytearray(open(blob, "rb").read())

    def check(b, name):
        p = str(d / name)
        open(p, "wb").write(bytes(b))
        with pytest.raises(bbh.BBHError) as e:
            bbh.blob_check(p)
        assert e.value.code == -4
        return str(e.value)

    assert "truncated" in check(raw[:-100], "short.bbhw")
    bad = bytearray(raw)
    bad[-1000] ^= 0x40
    assert "checksum" in check(bad, "flip.bbhw")
    bad = bytearray(raw)
    bad[0:4] = b"XXXX"
    assert "magic" in check(bad, "magic.bbhw")
    os.remove(str(d / "weights" / "encoder.layer.5.output.dense.bias.bin"))
    with pytest.raises(bbh.BBHError) as e:
        bbh.pack_weights(str(d / "weights"), 6, str(d / "x.bbhw"))
    assert e.value.code == -4
