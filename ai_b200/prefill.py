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
