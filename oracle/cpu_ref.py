"""The reference's CPU decode path restated in Numba (TEST / BASELINE INFRASTRUCTURE ONLY; see oracle/__init__.py).

What `bench.py` times as the CPU baseline (its `cpu_baseline` leg and `--impl reference`): the reference runs layers
it does not keep on the GPU with the Numba kernels of `ramvi/engine/ramvi_engine/cpu/cpu_layer.py` on bf16 weights
(`CpuLayer.__call__` :155-175: rms_rows :47-56, matmat16 :35-44 for q/k/v, qk_rope_attn :59-123, matmat16 o,
rms_rows, matmat16 gate/up, silu_mul :126-132, matmat16 down) and picks tokens from exact logits of the whole
vocabulary (`generation/head.py:19-26` exact_rows). This module restates those loops (the same arithmetic: fp32
sums over bf16 weights read as 2 bytes each, multi-threaded over output rows with `prange`; fastmath on the matrix
loops as the reference has it, off elsewhere) so the baseline runs on the GPU box's host cores, where the reference
package is not installed. The KV cache is fp32 as in `CpuLayer`.
"""
import math

import numba as nb
import numpy as np
from numba import types
from numba.extending import intrinsic


@intrinsic
def _f32_bits(typingctx, x):
    """Reinterpret a uint32 as fp32 (an LLVM bitcast; Numba has no scalar view)."""
    sig = types.float32(types.uint32)

    def codegen(context, builder, signature, args):
        return builder.bitcast(args[0], context.get_value_type(types.float32))
    return sig, codegen


@nb.njit(inline="always")
def bf16(u):
    return _f32_bits(np.uint32(u) << np.uint32(16))


@nb.njit(parallel=True, fastmath=True, cache=True, nogil=True)
def matmat16(W, X, Y, add):
    """Y[t] (+)= W X[t]; W [out, in] bf16 bits (uint16) -- cpu_layer.py:35-44."""
    n_out, n_in = W.shape
    T = X.shape[0]
    for o in nb.prange(n_out):
        for t in range(T):
            s = np.float32(0.0)
            for i in range(n_in):
                s += bf16(W[o, i]) * X[t, i]
            if add:
                Y[t, o] += s
            else:
                Y[t, o] = s


@nb.njit(fastmath=False, cache=True, nogil=True)
def rms_rows(X, w, out, eps):
    """cpu_layer.py:47-56."""
    T, D = X.shape
    for t in range(T):
        s = np.float32(0.0)
        for i in range(D):
            s += X[t, i] * X[t, i]
        r = np.float32(1.0) / np.float32(math.sqrt(s / np.float32(D) + np.float32(eps)))
        for i in range(D):
            out[t, i] = w[i] * (X[t, i] * r)


@nb.njit(parallel=True, fastmath=False, cache=True, nogil=True)
def silu_mul(GU, M, FF):
    """cpu_layer.py:126-132."""
    for t in nb.prange(GU.shape[0]):
        for i in range(FF):
            g = GU[t, i]
            M[t, i] = g / (np.float32(1.0) + np.float32(math.exp(-g))) * GU[t, FF + i]


@nb.njit(cache=True, nogil=True)
def _norm_rope(v, w, p, inv, eps, out):
    HD = v.shape[0]
    half = HD // 2
    s = np.float32(0.0)
    for d in range(HD):
        s += v[d] * v[d]
    r = np.float32(1.0) / np.float32(math.sqrt(s / np.float32(HD) + np.float32(eps)))
    for d in range(half):
        ang = np.float32(p) * inv[d]
        c, sn = np.float32(math.cos(ang)), np.float32(math.sin(ang))
        a = w[d] * (v[d] * r)
        b = w[d + half] * (v[d + half] * r)
        out[d] = a * c - b * sn
        out[d + half] = b * c + a * sn


@nb.njit(parallel=True, fastmath=False, cache=True, nogil=True)
def qk_rope_attn(QKV, qn, kn, inv, pos0, Kc, Vc, out, H, KV, HD, eps):
    """QK-RMSNorm + RoPE, K/V rows into the fp32 cache at pos0..pos0+T-1, attention of token t over 0..pos0+t
    (cpu_layer.py:59-123)."""
    T = QKV.shape[0]
    G = H // KV
    for t in range(T):
        p = pos0 + t
        for g in range(KV):
            _norm_rope(QKV[t, (H + g) * HD:(H + g + 1) * HD], kn, p, inv, eps, Kc[g, p])
            for d in range(HD):
                Vc[g, p, d] = QKV[t, (H + KV + g) * HD + d]
    for th in nb.prange(T * H):
        t, h = th // H, th % H
        g, p = h // G, pos0 + th // H
        q = np.empty(HD, np.float32)
        _norm_rope(QKV[t, h * HD:(h + 1) * HD], qn, p, inv, eps, q)
        scale = np.float32(1.0) / np.float32(math.sqrt(HD))
        n = p + 1
        sc = np.empty(n, np.float32)
        m = np.float32(-1e30)
        for j in range(n):
            s = np.float32(0.0)
            for d in range(HD):
                s += q[d] * Kc[g, j, d]
            s *= scale
            sc[j] = s
            m = max(m, s)
        l = np.float32(0.0)
        for j in range(n):
            sc[j] = np.float32(math.exp(sc[j] - m))
            l += sc[j]
        for d in range(HD):
            out[t, h * HD + d] = 0.0
        for j in range(n):
            w = sc[j] / l
            for d in range(HD):
                out[t, h * HD + d] += w * Vc[g, j, d]


@nb.njit(parallel=True, fastmath=False, cache=True, nogil=True)
def exact_rows(W, toks, rows, H, out):
    """Exact fp32 logits (head.py:19-26): fp32 products summed in column order."""
    for i in nb.prange(toks.shape[0]):
        s = np.float32(0.0)
        t, r = toks[i], rows[i]
        for d in range(H.shape[1]):
            s += bf16(W[t, d]) * H[r, d]
        out[i] = s


class CpuLayer:
    """One decoder layer on the host (CpuLayer, cpu_layer.py:135-175): weights as bf16 bits, fused
    qkv [(H+2KV)HD, D] and gu [2FF, D] (the engine's fused matrices), fp32 KV cache."""

    def __init__(self, qkv, o, gu, down, ln1, ln2, qn, kn, cfg, maxt):
        self.W = {"qkv": qkv, "o": o, "gu": gu, "down": down}
        self.s = {"ln1": ln1, "ln2": ln2, "qn": qn, "kn": kn}
        self.cfg = cfg
        self.K = np.zeros((cfg.KV, maxt, cfg.HD), np.float32)
        self.V = np.zeros_like(self.K)

    def __call__(self, X, pos0, inv):
        c, W, s = self.cfg, self.W, self.s
        T = X.shape[0]
        h = np.empty_like(X)
        rms_rows(X, s["ln1"], h, np.float32(c.eps))
        qkv = np.empty((T, (c.H + 2 * c.KV) * c.HD), np.float32)
        matmat16(W["qkv"], h, qkv, False)
        att = np.empty((T, c.H * c.HD), np.float32)
        qk_rope_attn(qkv, s["qn"], s["kn"], inv, pos0, self.K, self.V, att, c.H, c.KV, c.HD, np.float32(c.eps))
        matmat16(W["o"], att, X, True)
        rms_rows(X, s["ln2"], h, np.float32(c.eps))
        gu = np.empty((T, 2 * c.FF), np.float32)
        matmat16(W["gu"], h, gu, False)
        m = np.empty((T, c.FF), np.float32)
        silu_mul(gu, m, c.FF)
        matmat16(W["down"], m, X, True)
