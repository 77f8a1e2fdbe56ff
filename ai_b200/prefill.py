"""Whole-prompt prefill -- the reference's blocked prefill (`ramvi/engine/ramvi_engine/kernels/prefill.py`) on sm_100a.

Same names and argument meanings as the reference module:
  matrix(x, w, y, add=False)                  y (+)= x W^T for every prompt row (prefill.py:66-78). Here one
                                              tcgen05 GEMM launch decodes the 12-bit planes into the tensor
                                              cores' operand tiles; the reference decodes 512-row fp32 blocks
                                              (prefill_kernels.py:59-110) and multiplies them with mm_k (:8-27).
  attention(q, kc, vc, out, start, h, kv, hd) causal attention of the prompt rows over the KV cache: row i sees
                                              positions 0 .. start + i (prefill_kernels.py:30-56)
  layer(eng, l, x, start)                     one decoder layer over the whole prompt (prefill.py:81-121)
  enabled(n)                                  whether a prompt of n tokens takes this path (prefill.py:14-20)

`precision` (an addition): 3 (default) splits the activations into three bf16 parts, so the products are exact in
fp32 and the result has the accuracy of the reference's fp32 `mm_k`; 1 multiplies bf16 activations (one MMA per
step, three times the throughput, rel-err ~2^-9 per product).
"""
import ctypes as C
import os

import torch

from . import _lib, tkernels
from ._lib import ptr, stream_ptr

MIN_TOKENS = 17  # prompts up to 16 tokens run as one batched decode pass (the T <= 16 kernels)


def enabled(n=None):
    """True when a prompt of n tokens runs through the whole-prompt path (AIB_PREFILL=legacy turns it off)."""
    mode = os.environ.get("AIB_PREFILL", "blocked")
    if mode not in ("legacy", "blocked"):
        raise ValueError("AIB_PREFILL must be legacy or blocked")
    return mode == "blocked" and (n is None or n >= MIN_TOKENS)


def workspace(M, K, precision=3, device="cuda"):
    n = _lib.lib().aib_gemm_c12_workspace(M, K, precision)
    return torch.empty(max(n, 16), dtype=torch.uint8, device=device)


def matrix(x, w, y, add=False, precision=3, lnw=None, eps=1e-6, silu_input=False, gated=False, ws=None):
    """y[:M] (+)= xin(x[:M]) W^T, M = x.shape[0]. x fp32 [M, >=K] (>= 2K with silu_input: silu(x[:, :K]) *
    x[:, K:2K]); lnw: optional RMSNorm weights (bf16 [K]) applied to the rows first; gated: W's rows are (gate,
    up) pairs and y[:, i] = silu(gate_i) * up_i (y has N/2 columns)."""
    M, K, N = x.shape[0], int(w["K"]), int(w["N"])
    if x.dtype != torch.float32 or y.dtype != torch.float32 or x.stride(1) != 1 or y.stride(1) != 1:
        raise ValueError("matrix: x and y must be fp32 with contiguous rows")
    if y.shape[0] < M:
        raise ValueError("matrix: y has fewer rows than x")
    if ws is None:
        ws = workspace(M, K, precision, x.device)
    ymode = 3 if gated else (1 if add else 0)
    _lib.call("aib_gemm_c12", C.byref(w.desc()), ptr(x), M, x.stride(0), 2 if silu_input else 0,
              ptr(lnw.view(torch.int16)) if lnw is not None else None, float(eps), ptr(y), y.stride(0), ymode,
              precision, ptr(ws), ws.numel(), stream_ptr())
    return y


def attention(q, kc, vc, out, start, h, kv, hd):
    """Causal attention of the prompt rows q [n, h*hd] (normed + rotated) over the cache kc/vc [kv, maxt, hd] (bf16):
    row i sees positions 0 .. start + i (prefill_kernels.py:30-56, `attention`)."""
    n, maxt = q.shape[0], kc.shape[-2]
    _lib.call("aib_attn_prefill", ptr(q), ptr(kc.view(torch.int16)), ptr(vc.view(torch.int16)), ptr(out), n, int(start),
              h, kv, hd, maxt, float(hd ** -0.5), stream_ptr())
    return out


class Buffers:
    """Per-prompt work buffers of `layer` (allocated once per prefill call, reused by every layer)."""

    def __init__(self, eng, n):
        dev, H, KV, HD = eng.device, eng.H, eng.KV, eng.HD
        f = lambda c: torch.empty(n, c, device=dev)  # noqa: E731
        self.qkv, self.q, self.att = f((H + 2 * KV) * HD), f(H * HD), f(H * HD)
        self.mid = f(eng.FF if eng.gated else 2 * eng.FF)
        kmax = max(int(c["K"]) for c in eng.W[0].values())
        self.ws = workspace(n, kmax, eng.prefill_precision, dev)


def layer(eng, l, x, start, bufs=None):
    """One decoder layer over the whole prompt (prefill.py:81-121): x [n, D] fp32 residual rows, updated in place;
    the layer's K/V rows are written to the cache at positions start .. start + n - 1. Tensor parallel: rank 0
    adds its partial residual update, the other ranks write theirs, and the engine's all-reduce sums them."""
    n = x.shape[0]
    b = bufs or Buffers(eng, n)
    W, s = eng.W[l], eng.small[l]
    kc, vc = eng.kv[l, 0], eng.kv[l, 1]
    H, KV, HD, pr = eng.H, eng.KV, eng.HD, eng.prefill_precision
    add = eng._add == 1
    matrix(x, W["qkv"], b.qkv, precision=pr, lnw=s["ln1"], eps=eng.eps, ws=b.ws)
    eng.pos.fill_(start)
    tkernels.qk_rope_cache(b.qkv, s["qn"], s["kn"], eng.inv, eng.pos, b.q, kc, vc, eng.maxt, eng.eps, H, KV, HD, n)
    attention(b.q, kc, vc, b.att, start, H, KV, HD)
    matrix(b.att, W["o"], x, add=add, precision=pr, ws=b.ws)
    eng._reduce(x)
    if eng.gated:  # rows interleaved (gate_i, up_i): the GEMM writes silu(gate) * up directly
        matrix(x, W["gu"], b.mid, precision=pr, lnw=s["ln2"], eps=eng.eps, gated=True, ws=b.ws)
        matrix(b.mid, W["down"], x, add=add, precision=pr, ws=b.ws)
    else:
        matrix(x, W["gu"], b.mid, precision=pr, lnw=s["ln2"], eps=eng.eps, ws=b.ws)
        matrix(b.mid, W["down"], x, add=add, precision=pr, silu_input=True, ws=b.ws)
    eng._reduce(x)
    return x
