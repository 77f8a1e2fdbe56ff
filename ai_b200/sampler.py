"""Device token sampler -- the reference's logits-in `_pick` (core/gengine.py:452-469) on one sm_100a kernel.

`pick(logits, temperature, top_p, rng, mask)` keeps the reference signature (rng: numpy Generator; it draws
exactly one `rng.random()` per sampled row, the same draw `Generator.choice(n, p)` makes, so a seeded rng
gives the reference's tokens). `sample(...)` adds top-k and repetition/presence/frequency penalties (no
reference counterpart; see aib_sample in include/ai_b200.h for the order of the steps).
"""
import numpy as np
import torch

from . import _lib
from ._lib import SampleParams, ptr, stream_ptr

PMAX = 4096


def params(temperature=0.0, top_k=0, top_p=1.0, repetition_penalty=1.0, presence_penalty=0.0,
           frequency_penalty=0.0):
    return SampleParams(float(temperature), int(top_k), float(top_p), float(repetition_penalty),
                        float(presence_penalty), float(frequency_penalty))


def workspace(B, V, device):
    """Scratch for the two-phase sampler path (slice partials + candidates); reuse it across calls."""
    n = _lib.lib().aib_sample_workspace(B, V)
    return torch.empty(max(n, 16), dtype=torch.uint8, device=device)


def sample_into(logits, out_ids, prm, u=None, prior=None, mask=None, B=None, ws=None):
    """Launch the sampler on rows [0, B) of logits [>=B, V] (fp32, CUDA) writing int64 ids into out_ids.
    u: float64 [B] CUDA tensor or None (greedy); prior: int32 [B, P] (-1 = empty); mask: int32 [B, ceil(V/32)];
    ws: uint8 workspace from `workspace(B, V)` (selects the multi-CTA path; None = one CTA per row)."""
    B = logits.shape[0] if B is None else B
    V = logits.shape[-1]
    ld = logits.stride(0) if logits.dim() > 1 else V
    n_prior = 0 if prior is None else prior.shape[-1]
    if prior is not None and prior.dtype != torch.int32:
        raise ValueError("prior ids must be int32")
    if mask is not None and (mask.dtype != torch.int32 or mask.shape[-1] != (V + 31) // 32):
        raise ValueError("mask must be int32 [B, ceil(V/32)]")
    _lib.call("aib_sample", ptr(logits), B, V, ld, prm, ptr(prior), n_prior, ptr(mask), ptr(u), ptr(out_ids),
              ptr(ws), 0 if ws is None else ws.numel(), stream_ptr())


def sample(logits, temperature=0.0, top_p=1.0, top_k=0, us=None, prior=None, mask=None, repetition_penalty=1.0,
           presence_penalty=0.0, frequency_penalty=0.0, two_phase=True):
    """Convenience: returns a list of token ids. `us`: per-row uniform draws (sequence or tensor)."""
    if logits.dim() == 1:
        logits = logits[None]
    B = logits.shape[0]
    dev = logits.device
    out = torch.empty(B, dtype=torch.int64, device=dev)
    u = None
    if temperature > 0:
        if us is None:
            raise ValueError("sampling needs uniform draws")
        u = torch.as_tensor(np.asarray(us, np.float64)).to(dev)
    prm = params(temperature, top_k, top_p, repetition_penalty, presence_penalty, frequency_penalty)
    ws = workspace(B, logits.shape[-1], dev) if two_phase else None
    sample_into(logits.contiguous(), out, prm, u, prior, mask, ws=ws)
    return out.tolist()


def pick(logits, temperature=0.0, top_p=1.0, rng=None, mask=None):
    """GGUFEngine._pick semantics (gengine.py:452-469): logits [T, V]; mask = xgrammar-style int32 bitmask."""
    if logits.dim() == 1:
        logits = logits[None]
    us = None
    if temperature > 0:
        rng = rng or np.random.default_rng()
        us = [rng.random() for _ in range(logits.shape[0])]
    return sample(logits, temperature, top_p, 0, us, None, mask)
