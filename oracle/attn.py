"""Norm / RoPE / attention oracle (TEST INFRASTRUCTURE ONLY; see oracle/__init__.py).

Follows `ramvi/engine/ramvi_engine/kernels/tkernels.py`:
  rmsg_k :216-225, qk_rope_cache_k :82-120, attn_k :123-150, rope_attn_k :164-213,
and `kernels/prefill_kernels.py` att_k :30-56 (causal block attention for prefill).
Elementwise math is fp32 like the reference; softmax-weighted sums are exact (float64) -- the reference's
online softmax equals the exact softmax up to fp32 rounding. K/V written to a bf16 cache are rounded to
bf16 exactly as `.to(KC.dtype.element_ty)` does (tkernels.py:188-190): round-to-nearest-even on a GPU
(`kv_round="rne"`, the default and the product's semantics); `kv_round="rtz"` reproduces the Triton
interpreter, which truncates, and is used only to pin this oracle against interpreter-made goldens.
"""
import numpy as np

from .codec import bf16_bits_to_f32, to_bf16_bits, round_bf16


def rmsg(x, w_bits, eps):
    """tkernels.py:216-225, rows of x [T, D]."""
    x = np.asarray(x, np.float32)
    v = (x * x).sum(-1, dtype=np.float32) / np.float32(x.shape[-1])
    r = (np.float32(1.0) / np.sqrt(v + np.float32(eps))).astype(np.float32)
    return (bf16_bits_to_f32(w_bits) * (x * r[..., None])).astype(np.float32)


def rope_inv(HD, theta):
    """RoPE inverse frequencies as the engine builds them (core/engine.py:204)."""
    return (1.0 / (np.float32(theta) ** (np.arange(0, HD, 2, dtype=np.float32) / np.float32(HD)))).astype(np.float32)


def _norm_rope(v, w_bits, c, s, eps):
    """QK-RMSNorm + half-split RoPE of one head vector (tkernels.py:94-106 / :176-184)."""
    HD = v.shape[-1]
    half = HD // 2
    a, b = v[..., :half], v[..., half:]
    rs = np.float32(1.0) / np.sqrt(((a * a).sum(-1, dtype=np.float32) + (b * b).sum(-1, dtype=np.float32))
                                   / np.float32(HD) + np.float32(eps))
    rs = np.float32(rs)
    w = bf16_bits_to_f32(w_bits)
    a = (w[:half] * (a * rs)).astype(np.float32)
    b = (w[half:] * (b * rs)).astype(np.float32)
    return np.concatenate([(a * c - b * s).astype(np.float32), (b * c + a * s).astype(np.float32)], -1)


def _angles(pos, inv):
    ang = (np.float32(pos) * inv).astype(np.float32)
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def _softmax_av(q, K, V, scale):
    sc = (K.astype(np.float64) @ q.astype(np.float64)) * float(scale)
    p = np.exp(sc - sc.max())
    return (p @ V.astype(np.float64)) / p.sum()


def rope_attn(qkv, qn_bits, kn_bits, inv, pos, kc_bits, vc_bits, H, KV, HD, eps, kv_round="rne"):
    """T=1 fused step (tkernels.py:164-213). Caches are uint16 bf16 bits [KV, maxt, HD], updated in place.
    Returns out fp32 [H*HD]."""
    qkv = np.asarray(qkv, np.float32)
    G = H // KV
    c, s = _angles(pos, inv)
    scale = np.float32(HD ** -0.5)
    out = np.zeros(H * HD, np.float32)
    for g in range(KV):
        k = _norm_rope(qkv[(H + g) * HD:(H + g + 1) * HD], kn_bits, c, s, eps)
        v = qkv[(H + KV + g) * HD:(H + KV + g + 1) * HD]
        kc_bits[g, pos] = to_bf16_bits(k, kv_round)
        vc_bits[g, pos] = to_bf16_bits(v, kv_round)
        Kp = bf16_bits_to_f32(kc_bits[g, :pos + 1])
        Vp = bf16_bits_to_f32(vc_bits[g, :pos + 1])
        for h in range(g * G, (g + 1) * G):
            q = _norm_rope(qkv[h * HD:(h + 1) * HD], qn_bits, c, s, eps)
            out[h * HD:(h + 1) * HD] = _softmax_av(q, Kp, Vp, scale)
    return out


def qk_rope_cache(qkv, qn_bits, kn_bits, inv, pos0, kc_bits, vc_bits, H, KV, HD, eps, kv_round="rne"):
    """Batched prologue (tkernels.py:82-120): returns Q [T, H*HD] and writes k, v rows pos0..pos0+T-1."""
    qkv = np.asarray(qkv, np.float32)
    T = qkv.shape[0]
    Q = np.zeros((T, H * HD), np.float32)
    for t in range(T):
        c, s = _angles(pos0 + t, inv)
        for h in range(H):
            Q[t, h * HD:(h + 1) * HD] = _norm_rope(qkv[t, h * HD:(h + 1) * HD], qn_bits, c, s, eps)
        for g in range(KV):
            k = _norm_rope(qkv[t, (H + g) * HD:(H + g + 1) * HD], kn_bits, c, s, eps)
            kc_bits[g, pos0 + t] = to_bf16_bits(k, kv_round)
            vc_bits[g, pos0 + t] = to_bf16_bits(qkv[t, (H + KV + g) * HD:(H + KV + g + 1) * HD], kv_round)
    return Q


def attn(Q, kc_bits, vc_bits, pos0, H, KV, HD):
    """Batched causal decode attention (tkernels.py:123-150): token t attends 0..pos0+t."""
    T = Q.shape[0]
    G = H // KV
    out = np.zeros((T, H * HD), np.float32)
    scale = HD ** -0.5
    for t in range(T):
        n = pos0 + t + 1
        for h in range(H):
            g = h // G
            out[t, h * HD:(h + 1) * HD] = _softmax_av(Q[t, h * HD:(h + 1) * HD], bf16_bits_to_f32(kc_bits[g, :n]),
                                                       bf16_bits_to_f32(vc_bits[g, :n]), scale)
    return out


def prefill_attention(Q, kc_bits, vc_bits, start, H, KV, HD):
    """Causal block attention of att_k (prefill_kernels.py:30-56): query i (position start+i) sees
    positions 0..start+i of the cache."""
    return attn(Q, kc_bits, vc_bits, start, H, KV, HD)


__all__ = ["rmsg", "rope_inv", "rope_attn", "qk_rope_cache", "attn", "prefill_attention", "round_bf16"]
