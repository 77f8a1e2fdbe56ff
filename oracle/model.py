"""Whole-model Qwen3 decode oracle (TEST INFRASTRUCTURE ONLY; see oracle/__init__.py).

Restates the reference engine's T=1 decode step, `Engine._gpu_layer` (`core/engine.py:329-341`) + the
final `rmsg_k` (:380) + `Head.pick` (`generation/head.py:59-88`), in numpy:
    x += o( rope_attn( qkv( rms(x, ln1) ) ) );  x += down( silu(g)*u ( gu( rms(x, ln2) ) ) )
with every matrix passed through the 12-bit codec (compress -> exact decode, `kernels/wcomp.py`), a bf16
KV cache (the reference kernels round the current K/V to the cache dtype, tkernels.py:187-190), and
greedy = smallest id among the maximal logits.

Logits: `exact_head=True` computes them as Head.pick does (exact_rows, head.py:19-26: fp32 products summed
in column order in fp32), which is what the reference's greedy and sampled picks use; the default keeps the
float64 dot products (a tighter reference for GEMV-based heads). `codec_roundtrip=False` skips the
encode/decode of the layer matrices (the codec is lossless, pinned separately) to save time on big models.
"""
import numpy as np

from . import codec, gemv, attn, sampler


class DecodeOracle:
    def __init__(self, cfg, layers_bits, emb_bits, head_bits, norm_bits, maxt, kv_round="rne", exact_head=False,
                 codec_roundtrip=True):
        """layers_bits: list of dicts (qkv, o, gu, down, ln1, ln2, qn, kn) of uint16 bf16 bits."""
        self.cfg, self.maxt, self.kv_round = cfg, maxt, kv_round
        dec = (lambda b: codec.dense_f32(codec.compress(b))) if codec_roundtrip else codec.bf16_bits_to_f32
        self.W = [{n: dec(lb[n]).astype(np.float64) for n in ("qkv", "o", "gu", "down")} for lb in layers_bits]
        self.small = [{n: lb[n] for n in ("ln1", "ln2", "qn", "kn")} for lb in layers_bits]
        self.emb = codec.bf16_bits_to_f32(emb_bits)
        self.exact_head = exact_head
        self.head32 = codec.bf16_bits_to_f32(head_bits)
        self.head = None if exact_head else self.head32.astype(np.float64)
        self.norm = norm_bits
        self.inv = attn.rope_inv(cfg.HD, cfg.theta)
        self.kc = [np.zeros((cfg.KV, maxt, cfg.HD), np.uint16) for _ in range(cfg.L)]
        self.vc = [np.zeros((cfg.KV, maxt, cfg.HD), np.uint16) for _ in range(cfg.L)]

    def exact_logits(self, h):
        """exact_rows (head.py:19-26) over every vocabulary row for one fp32 row h."""
        prod = self.head32 * np.asarray(h, np.float32)[None, :]
        return np.add.accumulate(prod, axis=1, dtype=np.float32)[:, -1].copy()

    def step(self, token, pos, logits=True):
        """One T=1 decode step at position pos; returns fp32 logits [V] (None if logits is False)."""
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
        if not logits:
            return None
        if self.exact_head:
            return self.exact_logits(h)
        return (self.head @ h.astype(np.float64)).astype(np.float32)

    def greedy(self, prompt, steps):
        """Feed the prompt one token at a time, then `steps` greedy tokens; returns (tokens, logits)."""
        toks, lgs = [], []
        seq = list(prompt)
        for p in range(len(prompt) + steps - 1):
            want = p >= len(prompt) - 1
            lg = self.step(seq[p], p, logits=want)
            if want:
                t = int(np.flatnonzero(lg == lg.max()).min())
                toks.append(t)
                lgs.append(lg)
                seq.append(t)
        return toks, np.stack(lgs)

    def sample(self, prompt, steps, temperature, top_k=0, top_p=1.0, seed=None):
        """Head.pick sampling (head.py:62-87) on exact logits with the sampler's steps (`sampler.sample_row`),
        one uniform draw per picked token from np.random.default_rng(seed) in order -- the draws the engine's
        generate() makes."""
        rng = np.random.default_rng(seed)
        toks = []
        seq = list(prompt)
        for p in range(len(prompt) + steps - 1):
            want = p >= len(prompt) - 1
            self.step(seq[p], p, logits=False)
            if want:
                lg = self.exact_logits(self.last_h)
                t = sampler.sample_row(lg, temperature, top_k, top_p, u=rng.random())
                toks.append(t)
                seq.append(t)
        return toks
