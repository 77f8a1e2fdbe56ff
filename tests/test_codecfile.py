"""On-disk codec format (`ai_b200.codecfile`), on the CPU: encoded planes survive a save / load round trip
bit for bit, metadata mismatches and damaged files are refused."""
import json
import struct

import pytest
import torch

from ai_b200 import codecfile, wcomp


def _mats():
    g = torch.Generator().manual_seed(3)
    a = (torch.randn(64, 512, generator=g) * 0.02)
    a[3, 7] = 1e20   # exceptions on both sides of the exponent window
    a[9, 100] = 1e-30
    b = torch.randn(32, 256, generator=g) * 0.02  # typically no exception at all
    return {"layers.0.qkv": wcomp.compress(a.bfloat16()), "head": wcomp.compress(b.bfloat16())}


def test_round_trip(tmp_path):
    mats = _mats()
    p = str(tmp_path / "codec.safetensors")
    codecfile.save(p, mats, {"model": "t", "tp": "1:0"})
    got = codecfile.load(p, "cpu", expect={"model": "t", "tp": "1:0"})
    assert set(got) == set(mats)
    for name, c in mats.items():
        for k in ("m8", "e4", "rp", "er", "ec", "ev"):
            assert torch.equal(got[name][k], c[k].cpu()), (name, k)
        for k in ("base", "N", "K", "CH"):
            assert int(got[name][k]) == int(c[k])
    assert int(mats["layers.0.qkv"]["ev"].numel()) >= 2
    assert codecfile.read_meta(p)["model"] == "t"


def test_metadata_mismatch_refused(tmp_path):
    p = str(tmp_path / "codec.safetensors")
    codecfile.save(p, _mats(), {"model": "t", "tp": "1:0"})
    with pytest.raises(ValueError):
        codecfile.load(p, "cpu", expect={"model": "other"})
    with pytest.raises(ValueError):
        codecfile.load(p, "cpu", expect={"tp": "2:1"})


def test_damaged_file_refused(tmp_path):
    p = str(tmp_path / "codec.safetensors")
    codecfile.save(p, _mats(), {})
    with open(p, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
        rest = f.read()
    del header["head.e4"]  # a plane missing
    hb = json.dumps(header).encode()
    with open(p, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        f.write(rest)
    with pytest.raises(ValueError):
        codecfile.load(p, "cpu")
