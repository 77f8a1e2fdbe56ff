"""Token sampler oracle (TEST INFRASTRUCTURE ONLY; see oracle/__init__.py).

Reference semantics (pinned by golden vectors from the reference itself):
  * `pick` = GGUFEngine._pick (`ramvi/engine/ramvi_engine/core/gengine.py:452-469`) with the optional
    xgrammar bitmask of `Constraint.apply` (`generation/constrain.py:146-148`; int32 words, bit j of word w
    is token 32w+j, 1 = allowed, disallowed -> -inf): greedy = max with the first index on ties; sampling =
    softmax(l.double()/T), descending sort, keep where the exclusive cumsum < top_p, renormalise,
    `rng.choice`, here with a fixed uniform u: numpy's `Generator.choice(n, p)` returns
    searchsorted(cumsum(p)/cumsum[-1], u, 'right').
  * `head_pick` = Head.pick (`generation/head.py:59-88`) on exact logits.

Extension (PARITY UNPINNED -- the reference rejects these parameters, `server/validation.py:78-85`):
`sample` adds, in this order before the steps above: repetition penalty over the set of prior ids (HF
convention: l < 0 -> l * r, else l / r), presence/frequency penalties (OpenAI convention:
l -= f * count + p * [count > 0]), the bitmask, temperature, then top-k (keep every z >= the k-th largest,
HF TopKLogitsWarper convention) before top-p. With top_k <= 0 and no penalties it is exactly `pick`.
"""
import numpy as np


def apply_bitmask(l, mask_words):
    V = l.shape[-1]
    idx = np.arange(V)
    w = np.asarray(mask_words).view(np.uint32)
    allowed = ((w[..., idx >> 5] >> (idx & 31).astype(np.uint32)) & 1).astype(bool)
    return np.where(allowed, l, np.float32(-np.inf)).astype(np.float32)


def _choice_fixed_u(pr, u):
    cdf = np.cumsum(pr)
    cdf = cdf / cdf[-1]
    return min(int(np.searchsorted(cdf, u, side="right")), len(pr) - 1)


def pick_row(l, temperature, top_p, u):
    """One row of GGUFEngine._pick (gengine.py:452-469) with a fixed uniform u."""
    l = np.asarray(l, np.float32)
    if temperature <= 0:
        return int(np.argmax(l))            # torch .max(-1): first maximal index
    z = l.astype(np.float64) / temperature
    z = z - z.max()
    p = np.exp(z)
    p = p / p.sum()
    order = np.argsort(-p, kind="stable")
    sp = p[order]
    keep = (np.cumsum(sp) - sp) < top_p
    sp = sp * keep
    pr = sp / sp.sum()
    return int(order[_choice_fixed_u(pr, u)])


def pick(logits, temperature, top_p, us, mask=None):
    logits = np.asarray(logits, np.float32)
    if mask is not None:
        logits = apply_bitmask(logits, mask)
    return [pick_row(logits[b], temperature, top_p, us[b]) for b in range(logits.shape[0])]


def head_pick(exact, temperature, top_p, u):
    """Head.pick (head.py:72-87) on exact logits of one row."""
    l = np.asarray(exact, np.float32).astype(np.float64)
    c = np.arange(len(l))
    if temperature <= 0:
        m = l.max()
        return int(c[l == m].min())
    z = (l - l.max()) / temperature
    p = np.exp(z)
    p /= p.sum()
    o = np.argsort(-p, kind="stable")
    cs = np.cumsum(p[o])
    keep = o[:int(np.searchsorted(cs, top_p) + 1)]
    pk = p[keep] / p[keep].sum()
    return int(c[keep[_choice_fixed_u(pk, u)]])


def penalize(l, prior_ids, rep=1.0, presence=0.0, frequency=0.0):
    """Penalties of the extended sampler, fp32 arithmetic (see module docstring)."""
    l = np.array(l, np.float32, copy=True)
    V = l.shape[-1]
    ids = np.asarray(prior_ids, np.int64)
    ids = ids[(ids >= 0) & (ids < V)]
    if ids.size == 0:
        return l
    u, cnt = np.unique(ids, return_counts=True)
    v = l[u]
    if rep != 1.0:
        v = np.where(v < 0, v * np.float32(rep), v / np.float32(rep)).astype(np.float32)
    if presence != 0.0 or frequency != 0.0:
        t = (cnt.astype(np.float32) * np.float32(frequency) + np.float32(presence)).astype(np.float32)
        v = (v - t).astype(np.float32)
    l[u] = v
    return l


def sample_row(l, temperature=1.0, top_k=0, top_p=1.0, rep=1.0, presence=0.0, frequency=0.0,
               prior_ids=(), mask_words=None, u=0.5):
    """Extended sampler for one row (see module docstring for the order of the steps)."""
    l = penalize(l, prior_ids, rep, presence, frequency)
    if mask_words is not None:
        l = apply_bitmask(l, mask_words)
    if temperature <= 0:
        return int(np.argmax(l))
    z = l.astype(np.float64) / temperature
    if 0 < top_k < len(z):
        kth = np.partition(z, len(z) - top_k)[len(z) - top_k]
        z = np.where(z >= kth, z, -np.inf)
    z = z - z.max()
    p = np.exp(z)
    p = p / p.sum()
    order = np.argsort(-p, kind="stable")
    sp = p[order]
    keep = (np.cumsum(sp) - sp) < top_p
    sp = sp * keep
    pr = sp / sp.sum()
    return int(order[_choice_fixed_u(pr, u)])
