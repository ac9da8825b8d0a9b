"""GGUF load path (btf_gguf_*): the library's own reader against a file written
by the reference's GGUF writer (tests/golden/tiny_ptq.gguf, made by
tests/golden/make_gguf.py with bd::GgufWriter), malformed-file rejection, and
(-m gpu) PTQ1_0 -> panels on the device equal to the host repack twin."""
import hashlib
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN

META = json.load(open(os.path.join(GOLDEN, "MANIFEST_GGUF.json")))
PATH = os.path.join(GOLDEN, META["file"])


def test_fixture_checksum():
    assert hashlib.sha256(open(PATH, "rb").read()).hexdigest() == META["sha256"]


def test_reader_tensor_table_and_data(btf):
    with btf.GgufFile(PATH) as g:
        assert len(g) == len(META["tensors"])
        for i, t in enumerate(META["tensors"]):
            assert g.find(t["name"]) == i
            info = g.tensor(i)
            assert info["name"] == t["name"] and info["ne"] == [t["ne0"], t["ne1"]] and info["type"] == t["type"]
            assert info["bytes"] == t["bytes"]
            assert hashlib.sha256(g.data(i).tobytes()).hexdigest() == t["sha256"]
        assert g.find("no.such.tensor") == -1


def test_ptq_tensor_repacks_like_reference(btf, orc):
    import oracle
    import synth

    with btf.GgufFile(PATH) as g:
        for t in META["tensors"]:
            if t["type"] != btf.PTQ1_0:
                continue
            K, N = t["ne0"], t["ne1"]
            src = g.data(g.find(t["name"])).reshape(N, K // 128 * 28)
            assert np.array_equal(src, synth.ternary_ptq(N, K, seed=t["seed"]))
            codes, scales = oracle.panel_decode(btf.repack_panels_host(src, N, K), N, K)[:2]
            c_ref, s_ref = orc.repack_t2(src, N, K)
            assert np.array_equal(codes, c_ref) and np.array_equal(scales, s_ref)


def test_reader_rejects_malformed_files(btf, tmp_path):
    data = open(PATH, "rb").read()
    cases = {"missing": None, "truncated": data[:300], "magic": b"GGUX" + data[4:],
             "version": data[:4] + (9).to_bytes(4, "little") + data[8:],
             "tensor_beyond": data[:len(data) - 4096]}
    for name, blob in cases.items():
        p = tmp_path / f"{name}.gguf"
        if blob is not None:
            p.write_bytes(blob)
        with pytest.raises(RuntimeError):
            btf.GgufFile(str(p))


def _gguf_bytes(n_tensors, kvs):
    """A GGUF v3 header with the given tensor count and (key, type, value bytes) pairs, no tensor entries."""
    import struct

    out = b"GGUF" + struct.pack("<IQQ", 3, n_tensors, len(kvs))
    for key, typ, val in kvs:
        out += struct.pack("<Q", len(key)) + key.encode() + struct.pack("<I", typ) + val
    return out + bytes(64)


def test_reader_bounds_counts_alignment_and_float_metadata(btf, tmp_path):
    import struct

    bad = {"tensor_count": _gguf_bytes(1 << 23, []),
           "kv_count": b"GGUF" + struct.pack("<IQQ", 3, 0, 1 << 20) + bytes(64),
           "alignment": _gguf_bytes(0, [("general.alignment", 10, struct.pack("<Q", 1 << 40))])}
    for name, blob in bad.items():
        p = tmp_path / f"{name}.gguf"
        p.write_bytes(blob)
        with pytest.raises(RuntimeError, match="bad header|bad alignment"):
            btf.GgufFile(str(p))
    # float metadata that has no integer value (NaN, 1e30) is kept, not converted with undefined behaviour
    ok = tmp_path / "floats.gguf"
    ok.write_bytes(_gguf_bytes(0, [("a.nan", 6, struct.pack("<f", float("nan"))),
                                   ("a.big", 12, struct.pack("<d", 1e30))]))
    with btf.GgufFile(str(ok)) as g:
        assert len(g) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("staging", [1 << 20, 8 * 288])  # one chunk; one 8-row group per chunk
def test_load_panels_on_device_equals_host_twin(cuda, btf, staging):
    with btf.GgufFile(PATH) as g:
        for t in META["tensors"]:
            if t["type"] != btf.PTQ1_0:
                continue
            i = g.find(t["name"])
            pm = g.load_panels(i, staging_bytes=staging)
            host = btf.repack_panels_host(g.data(i).reshape(t["ne1"], -1), t["ne1"], t["ne0"])
            assert np.array_equal(pm.panels.cpu().numpy(), host)


def test_load_rows_rejects_bad_ranges(btf):
    # the row-range checks run before any device access
    L = btf.lib()
    with btf.GgufFile(PATH) as g:
        i = g.find("blk.0.ffn_up.weight")  # 37 rows
        for row0, rows in ((4, 8), (0, 0), (32, 8), (-8, 8), (40, 1)):  # row0 % 8, empty, past the end, negative
            assert L.btf_gguf_load_panels_rows(g.h, i, row0, rows, 256, 1 << 20, None) == 1, (row0, rows)
        j = g.find("output_norm.weight")  # not PTQ1_0
        assert L.btf_gguf_load_panels_rows(g.h, j, 0, 1, 256, 1 << 20, None) == 3


def test_load_rejects_a_ptq_width_not_a_multiple_of_128(btf, tmp_path):
    # a header that gives a PTQ1_0 tensor 64 columns (its data size becomes 0,
    # so the file opens): the loader refuses it before any device access
    import struct

    data = bytearray(open(PATH, "rb").read())
    name = b"blk.0.ffn_up.weight"
    at = data.index(struct.pack("<Q", len(name)) + name) + 8 + len(name)
    assert struct.unpack_from("<I", data, at)[0] == 2
    struct.pack_into("<Q", data, at + 4, 64)
    p = tmp_path / "narrow.gguf"
    p.write_bytes(bytes(data))
    L = btf.lib()
    with btf.GgufFile(str(p)) as g:
        i = g.find(name.decode())
        assert g.tensor(i)["ne"][0] == 64
        assert L.btf_gguf_load_panels_rows(g.h, i, 0, 8, 256, 1 << 20, None) == 1
        assert "multiple of 128" in L.btf_last_error().decode()


@pytest.mark.gpu
def test_load_rows_equals_the_full_load(cuda, btf):
    # one rank's shard: rows [8, 8 + n) of a 37-row tensor land in panel row
    # groups 0.. exactly as groups 1.. of the full load; a ragged tail (n = 29)
    # ends like the full matrix's last group
    with btf.GgufFile(PATH) as g:
        i = g.find("blk.0.ffn_up.weight")
        full = g.load_panels(i).panels.cpu().numpy()
        gbytes = btf.panel_bytes(8, 1152)  # one row group of all slices
        for row0, n in ((8, 16), (16, 8), (8, 29)):
            part = g.load_panels(i, rows=(row0, n)).panels.cpu().numpy()
            assert part.size == btf.panel_bytes(n, 1152)
            assert np.array_equal(part, full[row0 // 8 * gbytes:row0 // 8 * gbytes + part.size]), (row0, n)
