"""CPU checks of the convert host side: the blob format against the bytes the
reference writer produced, and argument / discovery errors (no GPU needed)."""
import ctypes as C
import os

import numpy as np

import ane_lm_cuda as A
from safetensors_util import blob_bytes, write_safetensors

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_blob_format_matches_reference_writer(oracle):
    g = np.load(os.path.join(GOLDEN, "convert_blobs.npz"))
    blobs = [k for k in g.files if k.startswith("blob:")]
    assert len(blobs) == 3
    raw = g["safetensors"].tobytes()
    import json
    import struct
    hl = struct.unpack("<Q", raw[:8])[0]
    hdr = json.loads(raw[8:8 + hl])
    data = raw[8 + hl:]
    for key in blobs:
        name = key[5:]
        a, b = hdr[name]["data_offsets"]
        bf = np.frombuffer(data[a:b], np.uint16)
        assert blob_bytes(oracle.bf16_to_f16(bf)) == g[key].tobytes(), name


def test_convert_errors_reported_on_host(ane, tmp_path):
    L = ane.lib()
    n = C.c_int64(-1)
    assert L.ane_cuda_convert_model(None, b"x", C.byref(n), None) == A.ERR_INVALID_ARG
    assert L.ane_cuda_write_ane_blobs(b"x", None, C.byref(n), None) == A.ERR_INVALID_ARG
    st = L.ane_cuda_convert_model(str(tmp_path / "missing").encode(), b"/tmp/x", C.byref(n), None)
    assert st == A.ERR_INVALID_ARG and b"not found" in L.ane_cuda_last_error()
    empty = tmp_path / "empty"
    empty.mkdir()
    st = L.ane_cuda_convert_model(str(empty).encode(), b"/tmp/x", C.byref(n), None)
    assert st == A.ERR_INVALID_ARG and b"no .safetensors" in L.ane_cuda_last_error()
    bad = tmp_path / "badidx"
    bad.mkdir()
    (bad / "model.safetensors.index.json").write_text('{"weight_map": {"a": "missing.safetensors"}}')
    st = L.ane_cuda_convert_model(str(bad).encode(), b"/tmp/x", C.byref(n), None)
    assert st == A.ERR_INVALID_ARG and b"missing shard" in L.ane_cuda_last_error()


def test_safetensors_util_roundtrip(tmp_path):
    p = tmp_path / "t.safetensors"
    write_safetensors(p, [("a.b", "BF16", np.arange(6, dtype=np.uint16).reshape(2, 3))], {"k": "v"})
    raw = p.read_bytes()
    import json
    import struct
    hl = struct.unpack("<Q", raw[:8])[0]
    hdr = json.loads(raw[8:8 + hl])
    assert hdr["a.b"]["shape"] == [2, 3] and hdr["__metadata__"] == {"k": "v"}
