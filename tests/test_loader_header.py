"""Host-side safetensors header parsing of ncmorph_b200.loader (the checks of
packages/safetensors/root.zig parse_header), on files written here."""
import json
import struct

import numpy as np
import pytest


def write_safetensors(path, tensors: dict, dtypes: dict):
    """tensors: name -> raw little-endian bytes; dtypes: name -> (dtype, shape)."""
    header, at, blobs = {}, 0, []
    for name, raw in tensors.items():
        dt, shape = dtypes[name]
        header[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [at, at + len(raw)]}
        at += len(raw)
        blobs.append(raw)
    hb = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for b in blobs:
            f.write(b)


def test_parse_header_offsets_and_validation(tmp_path):
    from ncmorph_b200 import loader
    a = np.arange(6, dtype=np.float32).reshape(2, 3)
    b = np.arange(4, dtype=np.uint16)
    p = tmp_path / "m.safetensors"
    write_safetensors(p, {"a": a.tobytes(), "b": b.tobytes()}, {"a": ("F32", (2, 3)), "b": ("BF16", (4,))})
    h = loader.parse_header(p)
    assert h.tensors["a"].shape == (2, 3) and h.tensors["b"].data_begin == 24
    assert h.offset(h.tensors["b"]) == 8 + h.header_len + 24
    bad = tmp_path / "bad.safetensors"
    write_safetensors(bad, {"a": a.tobytes()}, {"a": ("F32", (2, 2))})   # size mismatch
    with pytest.raises(ValueError):
        loader.parse_header(bad)
    with open(p, "ab") as f:
        f.write(b"\0")                                                    # trailing byte
    with pytest.raises(ValueError):
        loader.parse_header(p)
