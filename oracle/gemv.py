"""Codec GEMV/GEMM oracle (TEST INFRASTRUCTURE ONLY; see oracle/__init__.py).

Follows `ramvi/engine/ramvi_engine/kernels/wcomp.py`:
  _xin :57-64 (MODE 2 input silu(g)*u), gemvc1_k :67-112 (T=1, optional RMS prologue, exceptions),
  gemvc_tc_k :155-219 (T <= 16, split-K; numerically ~fp32 via the bf16x3 input split),
and `kernels/prefill.py:66-78` (`matrix`: Y (+)= X W^T in fp32 IEEE).
The dot products are accumulated in float64 and rounded to fp32 once (a tighter reference than any
fp32 summation order); the activation prologue is computed in fp32 exactly as the reference does.
"""
import numpy as np

from .codec import dense_f32, bf16_bits_to_f32


def silu_mul(g, u):
    """_xin MODE 2 (wcomp.py:59-62): g / (1 + exp(-g)) * u, in fp32."""
    g = np.asarray(g, np.float32)
    u = np.asarray(u, np.float32)
    with np.errstate(over="ignore"):
        return (g / (np.float32(1.0) + np.exp(-g)) * u).astype(np.float32)


def xin(x, K, mode, lnw_bits=None, eps=1e-6):
    """Effective input of gemvc1_k (wcomp.py:75-86): MODE 2 gating, then optional RMSNorm with LNW."""
    x = np.asarray(x, np.float32)
    xe = silu_mul(x[..., :K], x[..., K:2 * K]) if mode == 2 else x[..., :K].copy()
    if lnw_bits is not None:
        xr = x[..., :K]
        rs = (np.float32(1.0) / np.sqrt((xr * xr).sum(-1, dtype=np.float32) / np.float32(K) + np.float32(eps))).astype(np.float32)
        xe = (bf16_bits_to_f32(lnw_bits) * (xe * (rs[..., None] if xe.ndim > 1 else rs))).astype(np.float32)
    return xe


def gemvc1(x, c, y, mode, lnw_bits=None, eps=1e-6):
    """Returns the new y [N] (fp32) for y (+)= W xin(x) -- wcomp.py:67-112."""
    K = c["K"]
    W = dense_f32(c).astype(np.float64)
    acc = W @ xin(x, K, mode, lnw_bits, eps).astype(np.float64)
    y = np.asarray(y, np.float32)
    return acc.astype(np.float32) if mode == 0 else (y.astype(np.float64) + acc).astype(np.float32)


def gemvc_tc(X, c, Y, mode, T):
    """Returns new Y [16, N]; rows t < T updated (wcomp.py:155-219). X is [16, K or 2K]."""
    K = c["K"]
    W = dense_f32(c).astype(np.float64)
    Y = np.array(Y, np.float32, copy=True)
    xe = xin(X[:T], K, mode).astype(np.float64)
    acc = xe @ W.T
    Y[:T] = acc.astype(np.float32) if mode == 0 else (Y[:T].astype(np.float64) + acc).astype(np.float32)
    return Y


def matrix(x, c_or_w, y, add=False):
    """prefill.py:66-78: y (+)= x @ W^T for every row of x (fp32 in, fp32 out)."""
    W = dense_f32(c_or_w) if isinstance(c_or_w, dict) else np.asarray(c_or_w, np.float32)
    acc = np.asarray(x, np.float64) @ W.astype(np.float64).T
    y = np.asarray(y, np.float32)
    return (y.astype(np.float64) + acc).astype(np.float32) if add else acc.astype(np.float32)
