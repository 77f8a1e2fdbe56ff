"""Generate golden vectors from the reference implementation (karabilo214/AI, `ramvi/engine`).

Runs ONLY where the reference source tree is mounted (the build container); the fixtures it writes
(`tests/golden/*.npz`) are committed and are what the tests read everywhere else. Nothing here ships.

What is run, all from the reference's own code:
  * `kernels/wcomp.py`  compress (plain torch, CPU) and the Triton kernel gemvc1_k
  * `kernels/tkernels.py` rope_attn_k, qk_rope_cache_k, attn_k, rmsg_k
  * `kernels/prefill_kernels.py` decode_rows (dequant_k + exceptions_k), mm_k, att_k
  * `kernels/vocab8.py` vocab_a_k (called as `.fn` -- the autotuner needs a GPU driver)
  * `generation/head.py` Head tables (rebuilt on CPU with the same float64 arithmetic) and exact_rows
  * `core/gengine.py` GGUFEngine._pick and `generation/head.py` Head.pick with a fixed-uniform rng shim
  * a tiny Qwen3 decoded step by step with the reference's T=1 kernel sequence (`Engine._gpu_layer`,
    core/engine.py:329-341) on a bf16 KV cache, plus `core/reference.py` Reference.argmax math in fp32.
Triton kernels run with TRITON_INTERPRET=1 on CPU tensors. Two interpreter artefacts (Triton 3.6) shape the
fixtures: `tl.dot` on bf16 operands is wrong there (so gemvc_tc_k is not run), and fp32 -> bf16 `.to()`
truncates instead of rounding to nearest-even (so KV rows written by the attention kernels are truncated;
the oracle reproduces that with kv_round="rtz" when it is checked against these files).

Usage:  python tests/golden/make_golden.py [--only NAME]
"""
import os
import sys
import argparse
import hashlib

os.environ["TRITON_INTERPRET"] = "1"
REF = "/root/reference/ramvi/engine"
HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REF)
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import numpy as np
import torch

from ramvi_engine.kernels import wcomp, tkernels, prefill_kernels, vocab8  # noqa: E402

from ai_b200.model import CONFIGS, RandomWeights  # noqa: E402


def bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def cdict(prefix, c):
    return {f"{prefix}m8": c["m8"].numpy(), f"{prefix}e4": c["e4"].numpy(), f"{prefix}base": np.int32(c["base"]),
            f"{prefix}rp": c["rp"].numpy(), f"{prefix}er": c["er"].numpy(), f"{prefix}ec": c["ec"].numpy(),
            f"{prefix}ev": c["ev"].numpy()}


def digest(c):
    h = hashlib.sha256()
    for k in ("m8", "e4", "rp", "er", "ec", "ev"):
        h.update(c[k].contiguous().numpy().tobytes())
    h.update(str(int(c["base"])).encode())
    return h.hexdigest()


# ------------------------------------------------------------------------------------------- codec
def make_codec():
    out = {}
    cases = []
    # ET/legacy/test_prefill.py:25-30: seeds 7/43/109, injected out-of-window values
    for seed in (7, 43, 109):
        torch.manual_seed(seed)
        w = torch.randn(9, 512).bfloat16()
        w[3, 11] = 1e-30
        w[4, 92] = 1e20
        cases.append((f"prefill_s{seed}", w))
    torch.manual_seed(0)
    cases.append(("normal_64x1024", (torch.randn(64, 1024) * 0.02).bfloat16()))
    # special values: zeros, signed zero, subnormals, inf, nan, extremes
    torch.manual_seed(1)
    w = (torch.randn(16, 256) * 0.05).bfloat16()
    sv = torch.tensor([0.0, -0.0, float("inf"), float("-inf"), float("nan"), 3.3895e38, -3.3895e38,
                       1e-40, -1e-40, 9.2e-41, 1.0, -1.0, 2.0 ** -126, 65504.0, 1e-10, -7e10]).bfloat16()
    w[5, :16] = sv
    w[0, 255] = float("inf")
    w[15, 0] = -0.0
    cases.append(("special_16x256", w))
    # a whole row of exceptions, and a row with none
    torch.manual_seed(2)
    w = (torch.randn(8, 768) * 0.02).bfloat16()
    w[2] = (torch.randn(768) * 1e6).bfloat16()
    cases.append(("exc_row_8x768", w))
    # tie between two exponent windows: the first window must win (argmax of the sliding sums)
    e = torch.cat([torch.full((128,), 100), torch.full((128,), 130)]).int()
    b = (e << 7) | torch.randint(0, 128, (256,), generator=torch.Generator().manual_seed(3)).int()
    w = (b.to(torch.int16)).view(torch.bfloat16).reshape(1, 256)
    cases.append(("tie_1x256", w))
    # all-zero matrix (every element is an exception? exponent 0 -> window [0,14], none are)
    cases.append(("zeros_4x256", torch.zeros(4, 256).bfloat16()))
    names = []
    for name, w in cases:
        c = wcomp.compress(w)
        assert torch.equal(wcomp.decompress(c).view(torch.int16), w.view(torch.int16)) or \
            torch.isnan(w.float()).any(), name
        out[f"{name}/w"] = bits(w)
        out.update(cdict(f"{name}/", c))
        names.append(name)
    out["names"] = np.array(names)
    # BASELINE config 1 matrices (seed 0): digests only (too big to commit as raw arrays)
    torch.manual_seed(0)
    gate = (torch.randn(3072, 1024) * 0.02).bfloat16()
    up = (torch.randn(3072, 1024) * 0.02).bfloat16()
    down = (torch.randn(1024, 3072) * 0.02).bfloat16()
    big = {"cfg1_gate": gate, "cfg1_up": up, "cfg1_down": down, "cfg1_gu": torch.cat([gate, up])}
    for name, w in big.items():
        c = wcomp.compress(w)
        out[f"{name}/digest"] = np.array(digest(c))
        out[f"{name}/base"] = np.int32(c["base"])
        out[f"{name}/n_exc"] = np.int64(c["ev"].numel())
    np.savez_compressed(os.path.join(HERE, "codec.npz"), **out)
    print("codec:", names, {k: int(out[f'{k}/n_exc']) for k in big})


# -------------------------------------------------------------------------------------------- gemv
def make_gemv():
    out = {}
    names = []
    g = torch.Generator().manual_seed(11)
    for name, N, K, mode, rms in (("m0_rms", 64, 512, 0, True), ("m0", 48, 768, 0, False),
                                  ("m1", 64, 256, 1, False), ("m2", 32, 512, 2, False),
                                  ("m0_rms_exc", 40, 1024, 0, True), ("m2_exc", 24, 768, 2, False)):
        W = (torch.randn(N, K, generator=g) * 0.02).bfloat16()
        if "exc" in name:
            for (r, cc, v) in ((0, 3, 5.0), (7, 100, -1e-9), (7, 101, 3e3), (N - 1, K - 1, 40.0), (13, 0, -0.0)):
                W[r, cc] = v
        c = wcomp.compress(W)
        x = torch.randn(2 * K if mode == 2 else K, generator=g) * (3.0 if rms else 1.0)
        y0 = torch.randn(N, generator=g)
        lnw = (1 + 0.1 * torch.randn(K, generator=g)).bfloat16() if rms else None
        y = y0.clone()
        wcomp.gemvc1(x, c, y, mode, BN=8, w=4, lnw=lnw, eps=1e-6)
        out[f"{name}/w"] = bits(W)
        out[f"{name}/x"] = x.numpy()
        out[f"{name}/y0"] = y0.numpy()
        out[f"{name}/y"] = y.numpy()
        out[f"{name}/mode"] = np.int32(mode)
        if rms:
            out[f"{name}/lnw"] = bits(lnw)
        names.append(name)
    out["names"] = np.array(names)
    # The batched kernel gemvc_tc_k (wcomp.py:155-219) is NOT run here: under TRITON_INTERPRET=1 (Triton
    # 3.6) `tl.dot` on bf16 operands returns garbage (errors ~1e10-1e12 even for a plain bf16 x bf16 tile,
    # while fp32 tl.dot is correct), so its interpreter output cannot serve as a golden. Its oracle is
    # pinned per token through the gemvc1_k goldens above (same arithmetic at fp32 accuracy: the reference
    # splits x into three bf16 parts precisely to reproduce fp32, wcomp.py:131-140).
    np.savez_compressed(os.path.join(HERE, "gemv.npz"), **out)
    print("gemv:", names)


# ---------------------------------------------------------------------------------------- attention
def make_attn():
    out = {}
    g = torch.Generator().manual_seed(21)
    H, KV, HD, maxt, eps = 8, 2, 64, 128, 1e-6
    inv = 1.0 / (1e6 ** (torch.arange(0, HD, 2, dtype=torch.float32) / HD))
    for name, pos in (("p0", 0), ("p1", 1), ("p77", 77), ("p127", 127)):
        qkv = torch.randn((H + 2 * KV) * HD, generator=g) * 2.0
        qn = (1 + 0.1 * torch.randn(HD, generator=g)).bfloat16()
        kn = (1 + 0.1 * torch.randn(HD, generator=g)).bfloat16()
        KC = torch.randn(KV, maxt, HD, generator=g).bfloat16()
        VC = torch.randn(KV, maxt, HD, generator=g).bfloat16()
        k0, v0 = KC.clone(), VC.clone()
        o = torch.zeros(H * HD)
        P = torch.tensor([pos], dtype=torch.long)
        tkernels.rope_attn_k[(H,)](qkv, qn, kn, inv, P, KC, VC, o, maxt, eps, HD ** -0.5,
                                   NH=H, NKV=KV, HDIM=HD, half=HD // 2, BJ=64)
        d = {"qkv": qkv.numpy(), "qn": bits(qn), "kn": bits(kn), "kc0": bits(k0), "vc0": bits(v0),
             "kc": bits(KC), "vc": bits(VC), "out": o.numpy(), "pos": np.int64(pos)}
        out.update({f"{name}/{k}": v for k, v in d.items()})
    out["names"] = np.array(["p0", "p1", "p77", "p127"])
    out["inv"] = inv.numpy()
    out["cfg"] = np.array([H, KV, HD, maxt], np.int32)
    # batched: qk_rope_cache_k then attn_k (Engine._batch_layer, core/engine.py:344-356)
    T, pos = 5, 40
    qkv = torch.randn(T, (H + 2 * KV) * HD, generator=g)
    qn = (1 + 0.1 * torch.randn(HD, generator=g)).bfloat16()
    kn = (1 + 0.1 * torch.randn(HD, generator=g)).bfloat16()
    KC = torch.randn(KV, maxt, HD, generator=g).bfloat16()
    VC = torch.randn(KV, maxt, HD, generator=g).bfloat16()
    k0, v0 = KC.clone(), VC.clone()
    q = torch.zeros(T, H * HD)
    o = torch.zeros(T, H * HD)
    P = torch.tensor([pos], dtype=torch.long)
    tkernels.qk_rope_cache_k[(H + 2 * KV, T)](qkv, qn, kn, inv, P, q, KC, VC, maxt, eps,
                                              NH=H, NKV=KV, HDIM=HD, half=HD // 2)
    tkernels.attn_k[(H, T)](q, KC, VC, P, o, maxt, HD ** -0.5, G=H // KV, HDIM=HD, BJ=64, NHQ=H)
    d = {"qkv": qkv.numpy(), "qn": bits(qn), "kn": bits(kn), "kc0": bits(k0), "vc0": bits(v0), "kc": bits(KC),
         "vc": bits(VC), "q": q.numpy(), "out": o.numpy(), "pos": np.int64(pos), "T": np.int32(T)}
    out.update({f"batch/{k}": v for k, v in d.items()})
    # rmsg_k
    X = torch.randn(3, 300, generator=g) * 4
    Wn = (1 + 0.2 * torch.randn(300, generator=g)).bfloat16()
    O = torch.zeros(3, 300)
    tkernels.rmsg_k[(3,)](X, Wn, O, 1e-6, 300, DP=512)
    out.update({"rms/x": X.numpy(), "rms/w": bits(Wn), "rms/out": O.numpy()})
    np.savez_compressed(os.path.join(HERE, "attn.npz"), **out)
    print("attn: ok")


# ------------------------------------------------------------------------------------------ prefill
def make_prefill():
    out = {}
    g = torch.Generator().manual_seed(31)
    W = (torch.randn(40, 512, generator=g) * 0.02).bfloat16()
    W[3, 11] = 1e-30
    W[20, 500] = 1e20
    c = wcomp.compress(W)
    rows = prefill_kernels.decode_rows(c, 2, 37)
    out.update({"rows/w": bits(W), "rows/first": np.int32(2), "rows/last": np.int32(37), "rows/out": rows.numpy()})
    x = torch.randn(37, 512, generator=g)
    y = prefill_kernels.matmul(x, W.float())
    out.update({"mm/x": x.numpy(), "mm/y": y.numpy()})
    # causal block attention (att_k) over a bf16 cache, start > 0
    H, KV, HD, maxt, n, start = 4, 2, 64, 96, 37, 20
    q = torch.randn(n, H * HD, generator=g)
    KC = torch.randn(KV, maxt, HD, generator=g).bfloat16()
    VC = torch.randn(KV, maxt, HD, generator=g).bfloat16()
    o = torch.zeros(n, H * HD)
    prefill_kernels.attention(q, KC, VC, o, start, H, KV, HD)
    out.update({"att/q": q.numpy(), "att/kc": bits(KC), "att/vc": bits(VC), "att/out": o.numpy(),
                "att/cfg": np.array([H, KV, HD, maxt, n, start], np.int32)})
    np.savez_compressed(os.path.join(HERE, "prefill.npz"), **out)
    print("prefill: ok")


# --------------------------------------------------------------------------------------------- head
def head_tables(Wbf):
    """Head.__init__ (generation/head.py:29-50) arithmetic, on CPU in float64."""
    e = Wbf.double()
    am = e.abs().amax(1)
    s = (am / 127).float().double()
    s[s == 0] = 1.0
    q = torch.round(e / s[:, None]).clamp(-127, 127)
    d = e - q * s[:, None]
    return (q.to(torch.int8), s.float(), (d.abs().amax(1) * (1 + 1e-6)).float(),
            (d.norm(dim=1) * (1 + 1e-6)).float(), am.float())


def make_head():
    from ramvi_engine.generation.head import exact_rows
    out = {}
    g = torch.Generator().manual_seed(41)
    V, D, T = 300, 64, 3
    Wb = (torch.randn(V, D, generator=g) * 0.5).bfloat16()
    Wb[7] = 0  # zero row: scale 1
    Q, S, C1, C2, AM = head_tables(Wb)
    h = torch.randn(T, D, generator=g)
    HI = torch.zeros(16, V)
    LO = torch.full((16,), -float("inf"))
    vocab8.vocab_a_k.fn[(triton_cdiv(V, 32),)](h, Q, S, C1, C2, AM, HI, LO, T, V, D, BN=32, BK=64, KP=64)
    Wc = bits(Wb)
    toks = np.repeat(np.arange(V), T).astype(np.int64)
    rws = np.tile(np.arange(T), V).astype(np.int64)
    lg = np.empty(len(toks), np.float32)
    exact_rows(Wc, toks, rws, h.numpy(), lg)
    exact = np.zeros((T, V), np.float32)
    exact[rws, toks] = lg
    out.update({"w": Wc, "h": h.numpy(), "q": Q.numpy(), "s": S.numpy(), "c1": C1.numpy(), "c2": C2.numpy(),
                "am": AM.numpy(), "hi": HI[:T].numpy(), "lo": LO[:T].numpy(), "exact": exact})
    np.savez_compressed(os.path.join(HERE, "head.npz"), **out)
    print("head: ok")


def triton_cdiv(a, b):
    return (a + b - 1) // b


# ------------------------------------------------------------------------------------------ sampler
class FixedU:
    """rng shim: numpy Generator.choice(n, p) == searchsorted(cumsum(p)/cumsum[-1], u, 'right')."""

    def __init__(self, u):
        self.u = u

    def choice(self, n, p):
        cdf = np.cumsum(p)
        cdf /= cdf[-1]
        return int(np.searchsorted(cdf, self.u, side="right"))


def check_fixed_u_matches_numpy():
    rs = np.random.default_rng(123)
    for s in range(200):
        n = int(rs.integers(1, 50))
        p = rs.random(n) ** 3
        p /= p.sum()
        a = np.random.default_rng(s).choice(n, p=p)
        u = np.random.default_rng(s).random()
        assert a == FixedU(u).choice(n, p), (s, a)


def make_sampler():
    sys.path.insert(0, os.path.join(REF, "tests", "legacy"))
    from audit_support import definition
    from ramvi_engine.generation.constrain import Constraint
    check_fixed_u_matches_numpy()
    import types
    eng_cls = definition("gengine.py", "GGUFEngine", dict(Engine=object, GiB=2 ** 30, torch=torch, np=np))
    out = {}
    names = []
    g = torch.Generator().manual_seed(51)
    V = 1000
    for i, (B, temp, top_p, masked, scale) in enumerate(((3, 0.0, 1.0, False, 2.0), (3, 0.7, 0.8, False, 2.0),
                                                         (2, 1.3, 0.3, False, 2.0), (3, 0.7, 0.95, True, 3.0),
                                                         (2, 0.0, 1.0, True, 3.0), (1, 0.2, 1.0, False, 1.0),
                                                         (2, 2.0, 0.999, False, 0.5))):
        lg = torch.randn(B, V, generator=g) * scale
        if i == 0:
            lg[1, 17] = lg[1, 400] = lg[1].max() + 1.0  # tie: smallest id wins
        mask = None
        if masked:
            words = (V + 31) // 32
            mask = torch.randint(-2 ** 31, 2 ** 31 - 1, (B, words), generator=g, dtype=torch.int64).to(torch.int32)
            mask &= torch.randint(-2 ** 31, 2 ** 31 - 1, (B, words), generator=g, dtype=torch.int64).to(torch.int32)
        us = torch.rand(B, generator=g).double().numpy()
        ids = []
        for b in range(B):
            e = object.__new__(eng_cls)
            e.logits = lg[b:b + 1].clone()
            mk = mask[b:b + 1] if mask is not None else None
            if mk is not None:
                Constraint.apply(e.logits, mk)
            r = eng_cls._pick(e, 1, temp, top_p, FixedU(us[b]), None)
            ids.append(r[0])
        name = f"pick{i}"
        out.update({f"{name}/logits": lg.numpy(), f"{name}/u": us, f"{name}/temp": np.float64(temp),
                    f"{name}/top_p": np.float64(top_p), f"{name}/ids": np.array(ids, np.int64)})
        if mask is not None:
            out[f"{name}/mask"] = mask.numpy()
        names.append(name)
    out["names"] = np.array(names)
    # Head.pick sampling path (exact fp32 logits of the whole vocab, float64 softmax/top-p)
    from ramvi_engine.generation.head import Head
    hp = []
    for i, (temp, top_p) in enumerate(((0.0, 1.0), (0.7, 0.8), (1.0, 0.5), (0.3, 0.99))):
        Vh, D = 500, 32
        Wb = (torch.randn(Vh, D, generator=g) * 0.5).bfloat16()
        h = torch.randn(1, D, generator=g)
        hd = object.__new__(Head)
        hd.V, hd.D, hd.Wc = Vh, D, bits(Wb)
        hd.HI = torch.full((1, Vh), 1e30)
        hd.LO = torch.full((1,), -1e30)
        u = float(torch.rand(1, generator=g))
        r = hd.pick(h, 1, temp, top_p, FixedU(u), run_bounds=False)
        name = f"headpick{i}"
        out.update({f"{name}/w": bits(Wb), f"{name}/h": h.numpy(), f"{name}/u": np.float64(u),
                    f"{name}/temp": np.float64(temp), f"{name}/top_p": np.float64(top_p),
                    f"{name}/ids": np.array(r, np.int64)})
        hp.append(name)
    out["head_names"] = np.array(hp)
    np.savez_compressed(os.path.join(HERE, "sampler.npz"), **out)
    print("sampler:", names, hp)


# ------------------------------------------------------------------------------------- tiny model
def make_model(steps=12, prompt_len=6):
    """Reference T=1 decode sequence on a tiny random Qwen3 with a bf16 KV cache.

    Per layer, exactly Engine._gpu_layer (core/engine.py:329-341): gemvc1(qkv, RMS ln1) -> rope_attn_k ->
    gemvc1(o, MODE 1) -> gemvc1(gu, RMS ln2) -> gemvc1(down, MODE 2); then rmsg_k with the final norm and
    greedy Head.pick semantics (exact fp32 logits via exact_rows, smallest id among the maxima).
    """
    from ramvi_engine.generation.head import exact_rows
    cfg = CONFIGS["tiny"]
    rw = RandomWeights(cfg, seed=5, norm_noise=0.1)
    L, D, H, KV, HD, FF, V, eps = cfg.L, cfg.D, cfg.H, cfg.KV, cfg.HD, cfg.FF, cfg.V, cfg.eps
    inv = 1.0 / (cfg.theta ** (torch.arange(0, HD, 2, dtype=torch.float32) / HD))
    layers = [rw.layer(i) for i in range(L)]
    comp = [{n: wcomp.compress(lw[n]) for n in ("qkv", "o", "gu", "down")} for lw in layers]
    emb = rw.embedding()
    head = rw.head()
    hbits = bits(head)
    norm = rw.final_norm()
    maxt = 64
    KC = [torch.zeros(KV, maxt, HD).bfloat16() for _ in range(L)]
    VC = [torch.zeros(KV, maxt, HD).bfloat16() for _ in range(L)]
    prompt = [int(t) for t in torch.randint(0, V, (prompt_len,), generator=torch.Generator().manual_seed(6))]
    seq = list(prompt)
    logits_all = []
    toks = []
    for p in range(prompt_len + steps - 1):
        x = emb[seq[p]].float().clone()
        P = torch.tensor([p], dtype=torch.long)
        for l in range(L):
            W, lw = comp[l], layers[l]
            qkv = torch.zeros((H + 2 * KV) * HD)
            att = torch.zeros(H * HD)
            gu = torch.zeros(2 * FF)
            wcomp.gemvc1(x, W["qkv"], qkv, 0, BN=8, w=4, lnw=lw["ln1"], eps=eps)
            tkernels.rope_attn_k[(H,)](qkv, lw["qn"], lw["kn"], inv, P, KC[l], VC[l], att, maxt, eps, HD ** -0.5,
                                       NH=H, NKV=KV, HDIM=HD, half=HD // 2, BJ=64)
            wcomp.gemvc1(att, W["o"], x, 1, BN=8, w=4)
            wcomp.gemvc1(x, W["gu"], gu, 0, BN=8, w=4, lnw=lw["ln2"], eps=eps)
            wcomp.gemvc1(gu, W["down"], x, 2, BN=8, w=4)
        hb = torch.zeros(1, D)
        tkernels.rmsg_k[(1,)](x[None], norm, hb, eps, D, DP=256)
        lg = np.empty(V, np.float32)
        exact_rows(hbits, np.arange(V, dtype=np.int64), np.zeros(V, np.int64), hb.numpy(), lg)
        if p >= prompt_len - 1:
            m = lg.max()
            t = int(np.flatnonzero(lg == m).min())
            toks.append(t)
            logits_all.append(lg)
            seq.append(t)
        print(f"  step pos={p} done", flush=True)
    # Reference.argmax math (core/reference.py:25-61) in fp32 without a cache, teacher-forced on seq
    ref_tf = reference_argmax(cfg, layers, emb, head, norm, seq[:-1])
    out = {"prompt": np.array(prompt, np.int64), "tokens": np.array(toks, np.int64),
           "logits": np.stack(logits_all), "ref_fp32_argmax": np.array(ref_tf, np.int64),
           "seed": np.int64(5), "norm_noise": np.float64(0.1), "maxt": np.int64(maxt)}
    np.savez_compressed(os.path.join(HERE, "model_tiny.npz"), **out)
    print("model tiny tokens:", toks, "fp32 teacher-forced:", ref_tf[prompt_len - 1:])


def reference_argmax(cfg, layers, emb, head, norm, tokens):
    """`Reference.argmax` (core/reference.py:25-61) with the weights passed in, on CPU."""
    from ramvi_engine.core.reference import Reference
    H, KV, HD, eps, F = cfg.H, cfg.KV, cfg.HD, cfg.eps, cfg.FF
    T = len(tokens)
    rms = Reference.rms
    x = emb[torch.tensor(tokens)].float()
    inv = 1.0 / (cfg.theta ** (torch.arange(0, HD, 2, dtype=torch.int64).float() / HD))
    fr = torch.arange(T).float()[:, None] * inv[None]
    e = torch.cat([fr, fr], -1)
    cos, sin = e.cos(), e.sin()
    rot = lambda t: torch.cat([-t[..., HD // 2:], t[..., :HD // 2]], -1)  # noqa: E731
    mask = torch.full((T, T), float("-inf")).triu(1)
    for lw in layers:
        w = {k: v.float() for k, v in lw.items()}
        h = rms(x, w["ln1"], eps)
        qkv = h @ w["qkv"].T
        q = rms(qkv[:, :H * HD].view(T, H, HD), w["qn"], eps)
        k = rms(qkv[:, H * HD:(H + KV) * HD].view(T, KV, HD), w["kn"], eps)
        v = qkv[:, (H + KV) * HD:].view(T, KV, HD)
        q = q * cos[:, None] + rot(q) * sin[:, None]
        k = k * cos[:, None] + rot(k) * sin[:, None]
        k, v = k.repeat_interleave(H // KV, 1), v.repeat_interleave(H // KV, 1)
        a = torch.softmax((q.transpose(0, 1) @ k.permute(1, 2, 0)) * HD ** -0.5 + mask, -1)
        x = x + (a @ v.transpose(0, 1)).transpose(0, 1).reshape(T, H * HD) @ w["o"].T
        h = rms(x, w["ln2"], eps)
        gu = h @ w["gu"].T
        x = x + (torch.nn.functional.silu(gu[:, :F]) * gu[:, F:]) @ w["down"].T
    h = rms(x, norm.float(), eps)
    lg = h @ head.float().T
    return lg.argmax(-1).tolist()


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default=None)
    a = ap.parse_args()
    jobs = {"codec": make_codec, "gemv": make_gemv, "attn": make_attn, "prefill": make_prefill, "head": make_head,
            "sampler": make_sampler, "model": make_model}
    for k, f in jobs.items():
        if a.only is None or a.only == k:
            f()
