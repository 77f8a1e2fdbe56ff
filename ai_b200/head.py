"""Int8 vocabulary head -- the reference's `generation/head.py` `Head` on sm_100a kernels.

  Head(w, c12)          Head.__init__ (head.py:29-50): int8 copy Q [V, D] + S, C1, C2, AM [V] from the head's
                        bf16 weights `w`; `c12` is the same head in the 12-bit codec (`wcomp.compress`),
                        from which the exact candidate rows are decoded (lossless), so the bf16 head need
                        not stay resident
  .bounds(h, T)         Head.bounds / vocab_a_k (head.py:52-57, kernels/vocab8.py:19-44): HI [T, V], LO [T]
  .pick(h, T)           Head.pick with temperature 0 (head.py:59-88): exact fp32 logits of the candidates
                        HI >= LO, argmax with the smallest id on ties -> int64 ids [T] on the device

  exact_logits(h, c12, T, out)
                        the exact_rows arithmetic (head.py:19-26) for EVERY vocabulary row, as Head.pick does
                        for sampling (head.py:62-71): fp32 products, sequential fp32 sum in column order, on the
                        device from the 12-bit head; the sampler (`ai_b200.sampler`) then draws from them
"""
import ctypes as C

import torch

from . import _lib
from ._lib import ptr, stream_ptr


class Head:
    def __init__(self, w, c12, TM=16):
        if w.dtype != torch.bfloat16 or w.dim() != 2:
            raise ValueError("Head: w must be a bf16 [V, D] tensor")
        V, D = w.shape
        if (c12["N"], c12["K"]) != (V, D):
            raise ValueError("Head: the codec matrix must have the shape of w")
        if D % 16:
            raise ValueError("Head: D must be a multiple of 16")
        dev = w.device
        self.V, self.D, self.TM, self.c12 = V, D, TM, c12
        self.Q = torch.empty(V, D, dtype=torch.int8, device=dev)
        self.S, self.C1, self.C2, self.AM = (torch.empty(V, device=dev) for _ in range(4))
        w = w.contiguous()
        _lib.call("aib_head8_tables", ptr(w.view(torch.int16)), V, D, ptr(self.Q), ptr(self.S), ptr(self.C1),
                  ptr(self.C2), ptr(self.AM), stream_ptr())
        self.HI = torch.empty(TM, V, device=dev)
        self.LO = torch.full((TM,), -float("inf"), device=dev)
        self.out = torch.zeros(TM, dtype=torch.int64, device=dev)
        self.ws = torch.zeros(_lib.lib().aib_head8_workspace(V, D, TM), dtype=torch.uint8, device=dev)
        self._desc = c12.desc()

    def _h(self, h, T):
        if not (1 <= T <= self.TM) or h.dtype != torch.float32 or h.dim() != 2 or h.shape[1] != self.D:
            raise ValueError("Head: h must be fp32 [>=T, D] with 1 <= T <= TM")
        if h.stride(1) != 1:
            raise ValueError("Head: h rows must be contiguous")
        return h

    def bounds(self, h, T, k=1):
        """HI[:T], LO[:T] for rows h[:T] (on the device, graph-capturable). k > 1 (<= 32): LO bounds the k-th
        largest exact logit from below instead of the largest, so HI >= LO keeps every row of the exact top k."""
        h = self._h(h, T)
        if not 1 <= k <= 32:
            raise ValueError("Head.bounds: k must be in 1..32")
        _lib.call("aib_head8_bounds_topk", ptr(h), T, h.stride(0), ptr(self.Q), ptr(self.S), ptr(self.C1),
                  ptr(self.C2), ptr(self.AM), self.V, self.D, ptr(self.HI), self.V, ptr(self.LO), int(k), ptr(self.ws),
                  self.ws.numel(), stream_ptr())
        return self.HI[:T], self.LO[:T]

    def topk_logits(self, h, T, k, out):
        """out[:T, :V] = exact logits of every row that can be in the top k of h[:T] (the candidates of
        bounds(h, T, k)) and -inf elsewhere: what a top-k sampler needs, at the cost of the int8 pass plus the
        candidates' rows instead of the whole 12-bit head."""
        h = self._h(h, T)
        if out.dtype != torch.float32 or out.dim() != 2 or out.shape[0] < T or out.shape[1] < self.V or \
                out.stride(1) != 1:
            raise ValueError("Head.topk_logits: out must be fp32 [>=T, >=V] with contiguous rows")
        self.bounds(h, T, k)
        _lib.call("aib_head8_candidate_logits", ptr(h), T, h.stride(0), C.byref(self._desc), ptr(self.HI), self.V,
                  ptr(self.LO), ptr(out), out.stride(0), ptr(self.ws), self.ws.numel(), stream_ptr())
        return out[:T, :self.V]

    def pick(self, h, T, temperature=0.0, run_bounds=True, out=None):
        """Greedy ids for rows h[:T]: an int64 device tensor of length T (`out` if given, else a view of an
        internal buffer)."""
        if temperature > 0:
            raise NotImplementedError("Head.pick samples only greedily; use ai_b200.sampler for temperature > 0")
        h = self._h(h, T)
        if run_bounds:
            self.bounds(h, T)
        if out is not None and (out.dtype != torch.int64 or out.numel() < T or not out.is_contiguous()):
            raise ValueError("Head.pick: out must be a contiguous int64 tensor of >= T elements")
        dst = self.out if out is None else out
        _lib.call("aib_head8_greedy", ptr(h), T, h.stride(0), C.byref(self._desc), ptr(self.HI), self.V, ptr(self.LO),
                  ptr(dst), ptr(self.ws), self.ws.numel(), stream_ptr())
        return dst[:T]


def exact_logits(h, c12, T, out):
    """out[:T, :V] = exact fp32 logits of every row of the 12-bit head `c12` for h[:T] (fp32 [>=T, D], rows
    contiguous): the reference's exact_rows arithmetic (head.py:19-26) over the whole vocabulary."""
    if not (1 <= T <= 16) or h.dtype != torch.float32 or h.dim() != 2 or h.shape[1] != c12["K"] or h.stride(1) != 1:
        raise ValueError("exact_logits: h must be fp32 [>=T, D] with contiguous rows and 1 <= T <= 16")
    if out.dtype != torch.float32 or out.dim() != 2 or out.shape[0] < T or out.shape[1] < c12["N"] or out.stride(1) != 1:
        raise ValueError("exact_logits: out must be fp32 [>=T, >=V] with contiguous rows")
    _lib.call("aib_head_exact_logits", ptr(h), T, h.stride(0), C.byref(c12.desc()), ptr(out), out.stride(0),
              stream_ptr())
    return out[:T]
