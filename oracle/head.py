"""Vocabulary head oracle (TEST INFRASTRUCTURE ONLY; see oracle/__init__.py).

Follows `ramvi/engine/ramvi_engine/generation/head.py`:
  exact_rows :19-26 (exact fp32 logits: product rounded to fp32, sequential fp32 sum over d),
  Head.__init__ :29-50 (int8 copy + conservative error bounds, float64 arithmetic),
and `kernels/vocab8.py` vocab_a_k :19-44 (a = s*q.h; HI = a + B; LO = max(a - B)).
"""
import numpy as np

from .codec import bf16_bits_to_f32

SLACK = 2e-4  # vocab8.py:14


def tables(w_bits):
    """Head.__init__ arithmetic (head.py:37-48) in float64 -> (Q int8, S, C1, C2, AM) float32."""
    e = bf16_bits_to_f32(w_bits).astype(np.float64)
    am = np.abs(e).max(1)
    s = (am / 127).astype(np.float32).astype(np.float64)
    s[s == 0] = 1.0
    q = np.clip(np.round(e / s[:, None]), -127, 127)   # torch.round: half to even, as numpy
    d = e - q * s[:, None]
    return (q.astype(np.int8), s.astype(np.float32), (np.abs(d).max(1) * (1 + 1e-6)).astype(np.float32),
            (np.sqrt((d * d).sum(1)) * (1 + 1e-6)).astype(np.float32), am.astype(np.float32))


def bounds(h, Q, S, C1, C2, AM):
    """vocab_a_k (vocab8.py:19-44) for rows of h [T, D] -> HI [T, V], LO [T]."""
    h = np.asarray(h, np.float32)
    a = (Q.astype(np.float64) @ h.astype(np.float64).T).T * S[None].astype(np.float64)
    n1 = np.abs(h).sum(1, dtype=np.float64)[:, None]
    n2 = np.sqrt((h.astype(np.float64) ** 2).sum(1))[:, None]
    b = np.minimum(C2[None] * n2, C1[None] * n1) + SLACK * AM[None] * n1
    return (a + b).astype(np.float32), (a - b).max(1).astype(np.float32)


def exact_logits(w_bits, h):
    """exact_rows (head.py:19-26) for every vocab row: fp32 products, sequential fp32 sum."""
    W = bf16_bits_to_f32(w_bits)
    h = np.asarray(h, np.float32)
    out = np.empty((h.shape[0], W.shape[0]), np.float32)
    for r in range(h.shape[0]):
        prod = (W * h[r][None, :]).astype(np.float32)
        out[r] = np.add.accumulate(prod, axis=1, dtype=np.float32)[:, -1]
    return out


def logits_f64(w_bits, h):
    """High-precision logits (float64 dot products) -- the tolerance reference for GPU head GEMVs."""
    return (np.asarray(h, np.float64) @ bf16_bits_to_f32(w_bits).astype(np.float64).T)
