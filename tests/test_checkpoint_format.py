"""The optimizer-state file format on the CPU: the safetensors layout the
checkpoint module writes (length-prefixed JSON header padded to 8 bytes, raw
little-endian data at the declared offsets) and its reader."""
import json
import struct

import numpy as np
import pytest

from magicmindnet_b200 import checkpoint as C


def test_roundtrip_and_layout(tmp_path):
    p = tmp_path / "s.safetensors"
    t = {"b.m": np.arange(6, dtype=np.float32).reshape(2, 3),
         "a.velocity": np.array([1.5, -2.0], np.float32),
         "c.bits": np.array([0x3F80, 0x7F80], np.uint16),
         "d.count": np.array([7], np.int64)}
    C.write_safetensors(str(p), t, {"format": C.FORMAT, "adamw_step": 3})
    raw = p.read_bytes()
    (n,) = struct.unpack("<Q", raw[:8])
    assert n % 8 == 0
    header = json.loads(raw[8:8 + n])
    assert header["__metadata__"] == {"format": C.FORMAT, "adamw_step": "3"}
    # tensors in name order, back to back
    assert [k for k in header if k != "__metadata__"] == sorted(t)
    assert header["a.velocity"] == {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]}
    assert header["b.m"] == {"dtype": "F32", "shape": [2, 3], "data_offsets": [8, 32]}
    assert header["c.bits"]["dtype"] == "BF16"
    assert raw[8 + n:8 + n + 8] == struct.pack("<2f", 1.5, -2.0)
    got, meta = C.read_safetensors(str(p))
    assert meta["adamw_step"] == "3"
    for k, v in t.items():
        assert got[k].dtype == v.dtype and got[k].shape == v.shape
        np.testing.assert_array_equal(got[k], v)


def test_reader_rejects_truncated_files(tmp_path):
    p = tmp_path / "bad.safetensors"
    p.write_bytes(struct.pack("<Q", 1000) + b"{}")
    with pytest.raises(ValueError):
        C.read_safetensors(str(p))
    p.write_bytes(b"abc")
    with pytest.raises(ValueError):
        C.read_safetensors(str(p))


def test_reader_rejects_offsets_that_do_not_hold_the_shape(tmp_path):
    """A tensor whose data_offsets reach past the file, run backwards or span
    another byte count than its shape needs is refused by name."""
    p = tmp_path / "off.safetensors"
    C.write_safetensors(str(p), {"x.m": np.ones(4, np.float32)}, {"format": C.FORMAT})
    raw = p.read_bytes()
    (n,) = struct.unpack("<Q", raw[:8])
    header = json.loads(raw[8:8 + n])
    for offsets, shape in (([0, 32], [8]), ([8, 0], [4]), ([0, 12], [4]), ([-4, 12], [4])):
        h = dict(header)
        h["x.m"] = {"dtype": "F32", "shape": shape, "data_offsets": offsets}
        hb = json.dumps(h).encode()
        hb += b" " * ((8 - len(hb) % 8) % 8)
        p.write_bytes(struct.pack("<Q", len(hb)) + hb + raw[8 + n:])
        with pytest.raises(ValueError, match="x.m"):
            C.read_safetensors(str(p))
