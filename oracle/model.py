"""Whole-model Qwen3 decode oracle (TEST INFRASTRUCTURE ONLY; see oracle/__init__.py).

Restates the reference engine's T=1 decode step, `Engine._gpu_layer` (`core/engine.py:329-341`) + the
final `rmsg_k` (:380) + greedy `Head.pick` (`generation/head.py:72-79`), in numpy:
    x += o( rope_attn( qkv( rms(x, ln1) ) ) );  x += down( silu(g)*u ( gu( rms(x, ln2) ) ) )
with every matrix passed through the 12-bit codec (compress -> exact decode, `kernels/wcomp.py`), a bf16
KV cache (the reference kernels round the current K/V to the cache dtype, tkernels.py:187-190), and
greedy = smallest id among the maximal logits.
"""
import numpy as np

from . import codec, gemv, attn


class DecodeOracle:
    def __init__(self, cfg, layers_bits, emb_bits, head_bits, norm_bits, maxt, kv_round="rne"):
        """layers_bits: list of dicts (qkv, o, gu, down, ln1, ln2, qn, kn) of uint16 bf16 bits."""
        self.cfg, self.maxt, self.kv_round = cfg, maxt, kv_round
        self.W = [{n: codec.dense_f32(codec.compress(lb[n])).astype(np.float64) for n in ("qkv", "o", "gu", "down")}
                  for lb in layers_bits]
        self.small = [{n: lb[n] for n in ("ln1", "ln2", "qn", "kn")} for lb in layers_bits]
        self.emb = codec.bf16_bits_to_f32(emb_bits)
        self.head = codec.bf16_bits_to_f32(head_bits).astype(np.float64)
        self.norm = norm_bits
        self.inv = attn.rope_inv(cfg.HD, cfg.theta)
        self.kc = [np.zeros((cfg.KV, maxt, cfg.HD), np.uint16) for _ in range(cfg.L)]
        self.vc = [np.zeros((cfg.KV, maxt, cfg.HD), np.uint16) for _ in range(cfg.L)]

    def step(self, token, pos):
        """One T=1 decode step at position pos; returns fp32 logits [V] (float64 dot products)."""
        c = self.cfg
        x = self.emb[token].astype(np.float32).copy()
        for l in range(c.L):
            W, s = self.W[l], self.small[l]
            qkv = (W["qkv"] @ gemv.xin(x, c.D, 0, s["ln1"], c.eps).astype(np.float64)).astype(np.float32)
            att = attn.rope_attn(qkv, s["qn"], s["kn"], self.inv, pos, self.kc[l], self.vc[l], c.H, c.KV, c.HD, c.eps,
                                   self.kv_round)
            x = (x.astype(np.float64) + W["o"] @ att.astype(np.float64)).astype(np.float32)
            gu = (W["gu"] @ gemv.xin(x, c.D, 0, s["ln2"], c.eps).astype(np.float64)).astype(np.float32)
            mid = gemv.silu_mul(gu[:c.FF], gu[c.FF:])
            x = (x.astype(np.float64) + W["down"] @ mid.astype(np.float64)).astype(np.float32)
        h = attn.rmsg(x[None], self.norm, c.eps)[0]
        self.last_h = h
        return (self.head @ h.astype(np.float64)).astype(np.float32)

    def greedy(self, prompt, steps):
        """Feed the prompt one token at a time, then `steps` greedy tokens; returns (tokens, logits)."""
        toks, lgs = [], []
        seq = list(prompt)
        for p in range(len(prompt) + steps - 1):
            lg = self.step(seq[p], p)
            if p >= len(prompt) - 1:
                t = int(np.flatnonzero(lg == lg.max()).min())
                toks.append(t)
                lgs.append(lg)
                seq.append(t)
        return toks, np.stack(lgs)
