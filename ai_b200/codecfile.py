"""On-disk form of the 12-bit codec: encoded matrices saved next to a model so that a later load skips the
encoding pass (the reference encodes on the GPU at every load, `core/engine.py:223-224`).

One safetensors file holds any number of encoded matrices. Matrix `name` is stored as the tensors
`name.m8` (U8 [N, K]), `name.e4` (U8 [N, K/2]), `name.rp` (I32 [N+1]), `name.er`, `name.ec` (I32 [E]) and
`name.ev` (F32 [E]) -- the planes of `wcomp.compress` unchanged -- and its `base`, N, K and CH as the strings
`name.base`, `name.N`, `name.K`, `name.CH` in the file's `__metadata__`. The caller adds its own metadata
(model config, layout flags, tensor-parallel rank); `load` refuses a file whose metadata differ.
"""
import json
import os
import struct

import numpy as np
import torch

from .wcomp import C12

_PLANES = (("m8", "U8", torch.uint8), ("e4", "U8", torch.uint8), ("rp", "I32", torch.int32),
           ("er", "I32", torch.int32), ("ec", "I32", torch.int32), ("ev", "F32", torch.float32))
_NP = {"U8": np.uint8, "I32": np.int32, "F32": np.float32}
_SCALARS = ("base", "N", "K", "CH")


def save(path, mats, meta=None):
    """Write the C12 matrices `mats` ({name: C12}) and the string metadata `meta` to `path` (atomic rename)."""
    header, md, off = {}, {}, 0
    for k, v in (meta or {}).items():
        md[k] = str(v)
    order = []
    for name in sorted(mats):
        c = mats[name]
        for sfx in _SCALARS:
            md[f"{name}.{sfx}"] = str(int(c[sfx]))
        for plane, dt, _ in _PLANES:
            t = c[plane]
            n = t.numel() * t.element_size()
            header[f"{name}.{plane}"] = {"dtype": dt, "shape": list(t.shape), "data_offsets": [off, off + n]}
            order.append(t)
            off += n
    header["__metadata__"] = md
    hb = json.dumps(header).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for t in order:
            f.write(t.detach().contiguous().cpu().numpy().tobytes())
    os.replace(tmp, path)


def read_meta(path):
    """The file's string metadata (the caller's and the per-matrix scalars)."""
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        return json.loads(f.read(n)).get("__metadata__", {})


def load(path, device, expect=None):
    """{name: C12} on `device`. `expect`: metadata that must match the file's (else ValueError)."""
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
    base_off = 8 + n
    md = header.pop("__metadata__", {})
    for k, v in (expect or {}).items():
        if md.get(k) != str(v):
            raise ValueError(f"{path}: codec file made for {k}={md.get(k)!r}, this load needs {v!r}")
    names = sorted({k.rsplit(".", 1)[0] for k in header})
    out = {}
    for name in names:
        c = C12()
        for sfx in _SCALARS:
            if f"{name}.{sfx}" not in md:
                raise ValueError(f"{path}: matrix {name} lacks its {sfx}")
            c[sfx] = int(md[f"{name}.{sfx}"])
        for plane, dt, tdt in _PLANES:
            h = header.get(f"{name}.{plane}")
            if h is None or h["dtype"] != dt:
                raise ValueError(f"{path}: matrix {name} lacks its {plane} plane")
            a, b = h["data_offsets"]
            cnt = (b - a) // np.dtype(_NP[dt]).itemsize
            arr = np.fromfile(path, dtype=_NP[dt], count=cnt, offset=base_off + a).reshape(h["shape"])
            c[plane] = torch.from_numpy(arr).to(device)
        N, K = c["N"], c["K"]
        if tuple(c["m8"].shape) != (N, K) or tuple(c["e4"].shape) != (N, K // 2) or c["rp"].numel() != N + 1 \
                or not (c["er"].numel() == c["ec"].numel() == c["ev"].numel()):
            raise ValueError(f"{path}: matrix {name} has inconsistent planes")
        out[name] = c
    return out
