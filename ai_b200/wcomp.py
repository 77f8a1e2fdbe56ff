"""12-bit lossless bf16 codec and codec GEMV -- the reference's `kernels/wcomp.py` API on sm_100a kernels.

Same names, argument meanings and errors as `ramvi/engine/ramvi_engine/kernels/wcomp.py`:
  compress(W, CH=256)                      -> codec dict (:13-32); here a `C12` (a dict subclass)
  decompress(c)                            -> bf16 [N, K] (:35-45)
  gemvc1(x, c, y, mode, BN, w, lnw, eps)   -> y (+)= W xin(x) for one token (:118-126)
  gemvc_tc(x, c, y, mode, T, BN, w, S)     -> Y[t] (+)= W xin(X[t]) for T <= 16 tokens (:233-242)
plus `weight_rows` (prefill.py:23-42). BN / w / S are accepted for signature compatibility and ignored:
tile geometry is chosen per shape by the library (no autotuner, no `tune.json`).
Everything runs through `libai_b200.so`; there is no torch or CPU fallback for the compute.
"""
import ctypes as C

import torch

from . import _lib
from ._lib import C12Desc, ptr, stream_ptr

CH = 256


class C12(dict):
    """Encoded matrix: keys m8, e4, base, rp, er, ec, ev, N, K, CH (the reference dict layout)."""

    def desc(self):
        d = self.get("_desc")
        if d is None:
            has = self["ev"].numel() > 0
            d = C12Desc(self["m8"].data_ptr(), self["e4"].data_ptr(), self["rp"].data_ptr(),
                        self["er"].data_ptr() if has else None, self["ec"].data_ptr() if has else None,
                        self["ev"].data_ptr() if has else None, int(self["base"]), int(self["N"]), int(self["K"]),
                        int(self["CH"]), int(self["ev"].numel()))
            self["_desc"] = d
        return d

    @property
    def nbytes(self):
        return sum(self[k].numel() * self[k].element_size() for k in ("m8", "e4", "rp", "er", "ec", "ev"))

    def to(self, device):
        return C12({k: (v.to(device) if torch.is_tensor(v) else v) for k, v in self.items() if k != "_desc"})


def _check_w(W, CH_):
    if W.dim() != 2 or W.dtype != torch.bfloat16:
        raise ValueError("compress expects a 2-D bf16 tensor")
    N, K = W.shape
    if CH_ != CH or K % CH:
        raise ValueError(f"K={K} must be a multiple of {CH}")
    return N, K


def compress(W, CH=256):
    """W [N, K] bf16 -> C12. CUDA tensors are encoded on the device, CPU tensors by the host encoder."""
    N, K = _check_w(W, CH)
    W = W.contiguous()
    return _compress_device(W, N, K) if W.is_cuda else _compress_host(W, N, K)


def _compress_device(W, N, K):
    dev = W.device
    m8 = torch.empty(N, K, dtype=torch.uint8, device=dev)
    e4 = torch.empty(N, K // 2, dtype=torch.uint8, device=dev)
    rp = torch.empty(N + 1, dtype=torch.int32, device=dev)
    base_t = torch.empty(1, dtype=torch.int32, device=dev)
    ws = torch.empty(_lib.lib().aib_c12_encode_workspace(N), dtype=torch.uint8, device=dev)
    s = stream_ptr()
    _lib.call("aib_c12_encode_planes", ptr(W), N, K, ptr(m8), ptr(e4), ptr(rp), ptr(base_t), ptr(ws), ws.numel(), s)
    base = int(base_t.item())
    n = int(rp[N].item())
    er = torch.empty(n, dtype=torch.int32, device=dev)
    ec = torch.empty(n, dtype=torch.int32, device=dev)
    ev = torch.empty(n, dtype=torch.float32, device=dev)
    _lib.call("aib_c12_encode_exceptions", ptr(W), N, K, base, ptr(rp), ptr(er) if n else None,
              ptr(ec) if n else None, ptr(ev) if n else None, s)
    return C12(m8=m8, e4=e4, base=base, rp=rp, er=er, ec=ec, ev=ev, N=N, K=K, CH=CH)


def _compress_host(W, N, K):
    w16 = W.view(torch.int16)
    m8 = torch.empty(N, K, dtype=torch.uint8)
    e4 = torch.empty(N, K // 2, dtype=torch.uint8)
    rp = torch.empty(N + 1, dtype=torch.int32)
    base = C.c_int32(0)
    n = C.c_int64(0)
    rc = _lib.lib().aib_c12_encode_host(ptr(w16), N, K, ptr(m8), ptr(e4), ptr(rp), C.byref(base), C.byref(n), None,
                                        None, None, 0)
    if rc not in (_lib.AIB_OK, _lib.AIB_ESPACE):
        _lib.check(rc, "aib_c12_encode_host")
    er = torch.empty(n.value, dtype=torch.int32)
    ec = torch.empty(n.value, dtype=torch.int32)
    ev = torch.empty(n.value, dtype=torch.float32)
    if n.value:
        _lib.call("aib_c12_encode_host", ptr(w16), N, K, ptr(m8), ptr(e4), ptr(rp), C.byref(base), C.byref(n), ptr(er),
                  ptr(ec), ptr(ev), n.value)
    return C12(m8=m8, e4=e4, base=base.value, rp=rp, er=er, ec=ec, ev=ev, N=N, K=K, CH=CH)


def from_dict(c, device=None):
    """Wrap a reference-layout dict (torch tensors) as a C12, optionally moving it to `device`."""
    out = C12({k: c[k] for k in ("m8", "e4", "base", "rp", "er", "ec", "ev", "N", "K", "CH")})
    return out.to(device) if device is not None else out


def decompress(c):
    """Exact decode to bf16 [N, K] (reference wcomp.py:35-45)."""
    N, K = c["N"], c["K"]
    out = torch.empty(N, K, dtype=torch.bfloat16, device=c["m8"].device)
    _lib.call("aib_c12_decode", C.byref(c.desc()), 0, N, ptr(out), 1, stream_ptr())
    return out


def weight_rows(c, first, last):
    """Exact fp32 rows [first, last) (reference prefill.py:23-42 / decode_rows)."""
    out = torch.empty(last - first, c["K"], dtype=torch.float32, device=c["m8"].device)
    _lib.call("aib_c12_decode", C.byref(c.desc()), first, last, ptr(out), 0, stream_ptr())
    return out


def _chk(t, name):
    if not (t.is_cuda and t.dtype == torch.float32 and t.is_contiguous()):
        raise ValueError(f"{name} must be a contiguous fp32 CUDA tensor")


def gemv_workspace(cs, device):
    """Zero-filled workspace for `gemvc1(..., ws=...)` covering every matrix in `cs` (reused across calls on one
    stream: every call leaves it zeroed)."""
    n = max([_lib.lib().aib_gemv_c12_workspace(C.byref(c.desc()), 1) for c in cs] + [16])
    return torch.zeros(n, dtype=torch.uint8, device=device)


def gemvc1(x, c, y, mode, BN=None, w=None, lnw=None, eps=1e-6, ws=None):
    """y (+)= W xin(x) for one token (reference gemvc1, wcomp.py:118-126). ws: optional `gemv_workspace`
    (even split of the matrix over the SMs). mode 3 (no reference counterpart): W's rows are (gate, up) pairs
    and y[i] = silu((Wx)[2i]) * (Wx)[2i+1] -- see `interleave_gate_up`."""
    _chk(x, "x")
    _chk(y, "y")
    K = c["K"]
    if x.numel() < (2 * K if mode == 2 else K) or y.numel() < (c["N"] // 2 if mode == 3 else c["N"]):
        raise ValueError("gemvc1: x or y too small")
    if lnw is not None and lnw.dtype != torch.bfloat16:
        raise ValueError("lnw must be bf16")
    _lib.call("aib_gemv_c12", C.byref(c.desc()), ptr(x), ptr(y), 1, 0, 0, mode,
              ptr(lnw.view(torch.int16)) if lnw is not None else None, float(eps), ptr(ws),
              0 if ws is None else ws.numel(), stream_ptr())


def interleave_gate_up(gu):
    """[gate; up] ([2F, D], the reference's fused layout) -> rows (gate_0, up_0, gate_1, up_1, ...), the layout
    mode 3 expects. The encoder's per-matrix exponent base is unchanged (same set of values)."""
    F = gu.shape[0] // 2
    return gu.view(2, F, gu.shape[1]).transpose(0, 1).reshape(2 * F, gu.shape[1]).contiguous()


def gemvc_tc(x, c, y, mode, T, BN=None, w=None, S=None):
    """Y[t] (+)= W xin(X[t]), t < T <= 16 (reference gemvc_tc, wcomp.py:233-242). Row strides from x / y."""
    _chk(x, "x")
    _chk(y, "y")
    if not 1 <= T <= 16:
        raise ValueError("T must be in 1..16")
    if T == 1:
        return gemvc1(x[0] if x.dim() > 1 else x, c, y[0] if y.dim() > 1 else y, mode)
    xs = x.shape[-1]
    ys = y.shape[-1]
    _lib.call("aib_gemv_c12", C.byref(c.desc()), ptr(x), ptr(y), T, xs, ys, mode, None, 0.0, None, 0, stream_ptr())
