"""Norm / RoPE / attention launchers -- the reference's `kernels/tkernels.py` operations on sm_100a kernels.

  rmsg(x, w, out, eps)                                   rmsg_k (tkernels.py:216-225)
  rope_attn(qkv, qn, kn, inv, pos, kc, vc, out, ...)     rope_attn_k (:164-213), T = 1 fused step
  qk_rope_cache(qkv, qn, kn, inv, pos, q, kc, vc, ...)   qk_rope_cache_k (:82-120)
  attn(q, kc, vc, pos, out, ...)                         attn_k (:123-150) / prefill att_k
  embed(emb, ids, out)                                   Engine._emb (core/engine.py:388-390) on the device
KV caches are bf16 [KV, maxt, HD] (the reference HF engine allocates fp32, core/engine.py:234-235; the
kernels round the current k/v to the cache dtype either way, tkernels.py:187-190). `pos` is a device int64
scalar, so these launches can be captured once and replayed at any position.
"""
import torch

from . import _lib
from ._lib import ptr, stream_ptr

_WS = {}


def workspace(device, nbytes):
    """Caller-owned scratch of the attention kernels, per device (zero-filled once; the kernels re-zero their
    ticket counters). Calls that share it must not overlap on the GPU (one stream per device)."""
    key = str(device)
    buf = _WS.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        _WS[key] = buf
    return buf


def _b16(t):
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16)
    if t.dtype in (torch.int16, torch.uint16):
        return t
    raise ValueError("expected a bf16 tensor")


def rmsg(x, w, out, eps):
    T, D = x.shape
    _lib.call("aib_rmsnorm", ptr(x), ptr(_b16(w)), ptr(out), T, D, float(eps), stream_ptr())


def embed(emb, ids, out):
    V, D = emb.shape
    _lib.call("aib_embed", ptr(_b16(emb)), ptr(ids), ids.numel(), D, V, ptr(out), stream_ptr())


def rope_attn(qkv, qn, kn, inv, pos, kc, vc, out, maxt, eps, scale, NH, NKV, HDIM, ws=None):
    n = _lib.lib().aib_attn_workspace(NH, NKV, HDIM, maxt, 1)
    buf = ws if ws is not None else workspace(qkv.device, n)
    _lib.call("aib_rope_attn_decode", ptr(qkv), ptr(_b16(qn)), ptr(_b16(kn)), ptr(inv), ptr(pos), ptr(_b16(kc)),
              ptr(_b16(vc)), ptr(out), NH, NKV, HDIM, maxt, float(eps), float(scale), ptr(buf), buf.numel(),
              stream_ptr())


def qk_rope_cache(qkv, qn, kn, inv, pos, q, kc, vc, maxt, eps, NH, NKV, HDIM, T):
    _lib.call("aib_qk_rope_cache", ptr(qkv), ptr(_b16(qn)), ptr(_b16(kn)), ptr(inv), ptr(pos), ptr(q), ptr(_b16(kc)),
              ptr(_b16(vc)), T, NH, NKV, HDIM, maxt, float(eps), stream_ptr())


def attn(q, kc, vc, pos, out, maxt, scale, NH, NKV, HDIM, T, ws=None):
    n = _lib.lib().aib_attn_workspace(NH, NKV, HDIM, maxt, T)
    buf = ws if ws is not None else workspace(q.device, n)
    _lib.call("aib_attn_cached", ptr(q), ptr(_b16(kc)), ptr(_b16(vc)), ptr(pos), ptr(out), T, NH, NKV, HDIM, maxt,
              float(scale), ptr(buf), buf.numel(), stream_ptr())
