"""Pin the CPU oracle against golden vectors produced by the reference itself (no GPU needed)."""
import hashlib

import numpy as np
import pytest

from conftest import golden, cases, cdict
from oracle import codec, gemv, attn, head, sampler


# ------------------------------------------------------------------------------------------ codec
@pytest.mark.parametrize("name", cases(golden("codec")))
def test_codec_compress_bit_exact(name):
    z = golden("codec")
    c = codec.compress(z[f"{name}/w"])
    ref = cdict(z, f"{name}/")
    assert c["base"] == ref["base"]
    for k in ("m8", "e4", "rp", "er", "ec"):
        np.testing.assert_array_equal(c[k], ref[k], err_msg=k)
    np.testing.assert_array_equal(c["ev"].view(np.uint32), ref["ev"].view(np.uint32))


@pytest.mark.parametrize("name", cases(golden("codec")))
def test_codec_roundtrip(name):
    z = golden("codec")
    w = z[f"{name}/w"]
    d = codec.decompress(cdict(z, f"{name}/"))
    f = codec.bf16_bits_to_f32(w)
    nan = np.isnan(f)
    np.testing.assert_array_equal(d[~nan], w[~nan])
    assert np.isnan(codec.bf16_bits_to_f32(d[nan])).all()


def _digest(c):
    h = hashlib.sha256()
    for k in ("m8", "e4", "rp", "er", "ec", "ev"):
        h.update(np.ascontiguousarray(c[k]).tobytes())
    h.update(str(int(c["base"])).encode())
    return h.hexdigest()


def test_codec_baseline_config1_digests():
    """BASELINE config 1 matrices (torch.manual_seed(0): gate, up [3072,1024], down [1024,3072], N(0,.02))."""
    torch = pytest.importorskip("torch")
    z = golden("codec")
    torch.manual_seed(0)
    gate = (torch.randn(3072, 1024) * 0.02).bfloat16()
    up = (torch.randn(3072, 1024) * 0.02).bfloat16()
    down = (torch.randn(1024, 3072) * 0.02).bfloat16()
    for name, w in (("cfg1_gate", gate), ("cfg1_up", up), ("cfg1_down", down), ("cfg1_gu", torch.cat([gate, up]))):
        c = codec.compress(w.view(torch.int16).numpy().view(np.uint16))
        assert c["base"] == int(z[f"{name}/base"])
        assert len(c["ev"]) == int(z[f"{name}/n_exc"])
        assert _digest(c) == str(z[f"{name}/digest"])


def test_codec_weight_rows_matches_reference_decode_rows():
    z = golden("prefill")
    c = codec.compress(z["rows/w"])
    out = codec.weight_rows(c, int(z["rows/first"]), int(z["rows/last"]))
    np.testing.assert_array_equal(out.view(np.uint32), z["rows/out"].view(np.uint32))


# ------------------------------------------------------------------------------------------- gemv
@pytest.mark.parametrize("name", cases(golden("gemv")))
def test_gemvc1_oracle(name):
    z = golden("gemv")
    c = codec.compress(z[f"{name}/w"])
    lnw = z[f"{name}/lnw"] if f"{name}/lnw" in z.files else None
    y = gemv.gemvc1(z[f"{name}/x"], c, z[f"{name}/y0"], int(z[f"{name}/mode"]), lnw, 1e-6)
    np.testing.assert_allclose(y, z[f"{name}/y"], rtol=2e-5, atol=2e-6)


@pytest.mark.parametrize("name", cases(golden("gemv")))
def test_gemvc_tc_oracle_per_token(name):
    """gemvc_tc_k cannot run under the Triton interpreter (bf16 tl.dot is broken there); its per-token math
    equals gemvc1_k's, so row t of the batched oracle must reproduce the gemvc1_k golden for that token."""
    z = golden("gemv")
    if f"{name}/lnw" in z.files:
        pytest.skip("the batched path has no RMS prologue (the engine runs rmsg_k first)")
    c = codec.compress(z[f"{name}/w"])
    x, y0, mode = z[f"{name}/x"], z[f"{name}/y0"], int(z[f"{name}/mode"])
    rng = np.random.default_rng(0)
    for t in (0, 3, 15):
        X = rng.standard_normal((16, x.shape[0])).astype(np.float32)
        Y = rng.standard_normal((16, y0.shape[0])).astype(np.float32)
        X[t], Y[t] = x, y0
        out = gemv.gemvc_tc(X, c, Y, mode, 16)
        np.testing.assert_allclose(out[t], z[f"{name}/y"], rtol=2e-5, atol=2e-6)


def test_prefill_matrix_oracle():
    z = golden("prefill")
    W = codec.bf16_bits_to_f32(z["rows/w"])
    y = gemv.matrix(z["mm/x"], W, np.zeros((37, 40), np.float32))
    np.testing.assert_allclose(y, z["mm/y"], rtol=1e-5, atol=1e-6)


# -------------------------------------------------------------------------------------- attention
@pytest.mark.parametrize("name", cases(golden("attn")))
def test_rope_attn_oracle(name):
    z = golden("attn")
    H, KV, HD, maxt = (int(v) for v in z["cfg"])
    kc, vc = z[f"{name}/kc0"].copy(), z[f"{name}/vc0"].copy()
    out = attn.rope_attn(z[f"{name}/qkv"], z[f"{name}/qn"], z[f"{name}/kn"], z["inv"], int(z[f"{name}/pos"]),
                         kc, vc, H, KV, HD, 1e-6, kv_round="rtz")
    np.testing.assert_allclose(out, z[f"{name}/out"], rtol=1e-4, atol=2e-5)
    # the written K/V rows are the interpreter's truncations (at most 1 ulp where fp32 sums differ)
    dk = np.abs(kc.astype(np.int32) - z[f"{name}/kc"].astype(np.int32))
    assert dk.max() <= 1 and (dk > 0).sum() <= 2
    np.testing.assert_array_equal(vc, z[f"{name}/vc"])


def test_batched_attn_oracle():
    z = golden("attn")
    H, KV, HD, maxt = (int(v) for v in z["cfg"])
    kc, vc = z["batch/kc0"].copy(), z["batch/vc0"].copy()
    pos = int(z["batch/pos"])
    Q = attn.qk_rope_cache(z["batch/qkv"], z["batch/qn"], z["batch/kn"], z["inv"], pos, kc, vc, H, KV, HD, 1e-6,
                           kv_round="rtz")
    np.testing.assert_allclose(Q, z["batch/q"], rtol=1e-5, atol=1e-6)
    dk = np.abs(kc.astype(np.int32) - z["batch/kc"].astype(np.int32))
    assert dk.max() <= 1 and (dk > 0).sum() <= 4
    np.testing.assert_array_equal(vc, z["batch/vc"])
    out = attn.attn(Q, z["batch/kc"], z["batch/vc"], pos, H, KV, HD)
    np.testing.assert_allclose(out, z["batch/out"], rtol=1e-4, atol=2e-5)


def test_rmsg_oracle():
    z = golden("attn")
    out = attn.rmsg(z["rms/x"], z["rms/w"], 1e-6)
    np.testing.assert_allclose(out, z["rms/out"], rtol=1e-6, atol=1e-6)


def test_prefill_attention_oracle():
    z = golden("prefill")
    H, KV, HD, maxt, n, start = (int(v) for v in z["att/cfg"])
    out = attn.prefill_attention(z["att/q"], z["att/kc"], z["att/vc"], start, H, KV, HD)
    np.testing.assert_allclose(out, z["att/out"], rtol=1e-4, atol=2e-5)


# ------------------------------------------------------------------------------------------- head
def test_head_tables_and_bounds():
    z = golden("head")
    Q, S, C1, C2, AM = head.tables(z["w"])
    np.testing.assert_array_equal(Q, z["q"])
    np.testing.assert_array_equal(S, z["s"])
    np.testing.assert_allclose(C1, z["c1"], rtol=1e-7)
    np.testing.assert_allclose(C2, z["c2"], rtol=1e-6)
    np.testing.assert_array_equal(AM, z["am"])
    HI, LO = head.bounds(z["h"], Q, S, C1, C2, AM)
    np.testing.assert_allclose(HI, z["hi"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(LO, z["lo"], rtol=1e-5, atol=1e-5)
    ex = head.exact_logits(z["w"], z["h"])
    np.testing.assert_array_equal(ex, z["exact"])
    # the bounds are conservative: exact logits lie in [a - B, a + B]
    assert (ex <= HI + 1e-6).all()


# ---------------------------------------------------------------------------------------- sampler
@pytest.mark.parametrize("name", cases(golden("sampler")))
def test_pick_matches_reference(name):
    z = golden("sampler")
    mask = z[f"{name}/mask"] if f"{name}/mask" in z.files else None
    ids = sampler.pick(z[f"{name}/logits"], float(z[f"{name}/temp"]), float(z[f"{name}/top_p"]), z[f"{name}/u"], mask)
    np.testing.assert_array_equal(ids, z[f"{name}/ids"])


@pytest.mark.parametrize("name", cases(golden("sampler"), "head_names"))
def test_head_pick_matches_reference(name):
    z = golden("sampler")
    ex = head.exact_logits(z[f"{name}/w"], z[f"{name}/h"])[0]
    t = sampler.head_pick(ex, float(z[f"{name}/temp"]), float(z[f"{name}/top_p"]), float(z[f"{name}/u"]))
    assert t == int(z[f"{name}/ids"][0])
    # the logits-in sampler agrees with Head.pick away from measure-zero rounding boundaries
    assert sampler.pick_row(ex, float(z[f"{name}/temp"]), float(z[f"{name}/top_p"]), float(z[f"{name}/u"])) == t


def test_extended_sampler_reduces_to_pick():
    rng = np.random.default_rng(3)
    for _ in range(50):
        l = (rng.standard_normal(700) * 2).astype(np.float32)
        T, p, u = float(rng.uniform(0.1, 2)), float(rng.uniform(0.05, 1)), float(rng.random())
        assert sampler.sample_row(l, T, 0, p, u=u) == sampler.pick_row(l, T, p, u)


def test_extended_sampler_top_k_and_penalties():
    l = np.array([3.0, 2.0, 1.0, 0.5, -1.0], np.float32)
    # top_k 1 at T>0 always picks the max
    assert sampler.sample_row(l, 0.7, 1, 1.0, u=0.99) == 0
    # repetition penalty 100 on ids {0,1}: logits 0.03, 0.02 -> token 2 is the max
    assert sampler.sample_row(l, 0.0, 0, 1.0, rep=100.0, prior_ids=[0, 1, 1]) == 2
    # negative logits are multiplied: -1 * 0.5 = -0.5 ... with rep=0.5 (boost) token 4 -> -0.5
    pl = sampler.penalize(l, [4], rep=0.5)
    assert pl[4] == np.float32(-0.5)
    # frequency: count 2 * 1.5 + presence 1.0 = 4 off token 0
    pl = sampler.penalize(l, [0, 0, -1, 99], presence=1.0, frequency=1.5)
    assert pl[0] == np.float32(-1.0) and pl[1] == np.float32(2.0)
    # top-k keeps ties at the boundary
    l2 = np.array([1.0, 1.0, 1.0, 0.0], np.float32)
    picks = {sampler.sample_row(l2, 1.0, 2, 1.0, u=u) for u in np.linspace(0.01, 0.99, 30)}
    assert picks == {0, 1, 2}


def test_interpreter_truncates_bf16_but_rne_differs():
    """The goldens' KV rows are truncations of fp32 (interpreter behaviour); a GPU rounds to nearest-even."""
    z = golden("attn")
    H, KV, HD, maxt = (int(v) for v in z["cfg"])
    v = z["p0/qkv"][(H + KV) * HD:(H + KV + 1) * HD]
    np.testing.assert_array_equal(z["p0/vc"][0, 0], codec.f32_to_bf16_bits_rtz(v))
    assert (codec.f32_to_bf16_bits(v) != codec.f32_to_bf16_bits_rtz(v)).any()


def test_tiny_model_oracle_matches_reference_step_sequence():
    """The whole-model oracle reproduces the reference's T=1 kernel sequence (interpreter, rtz KV)."""
    from ai_b200.model import CONFIGS, RandomWeights
    from oracle.model import DecodeOracle
    import torch
    z = golden("model_tiny")
    cfg = CONFIGS["tiny"]
    rw = RandomWeights(cfg, seed=int(z["seed"]), norm_noise=float(z["norm_noise"]))
    b = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    layers = [{k: b(v) for k, v in rw.layer(i).items()} for i in range(cfg.L)]
    o = DecodeOracle(cfg, layers, b(rw.embedding()), b(rw.head()), b(rw.final_norm()), int(z["maxt"]), kv_round="rtz")
    toks, lg = o.greedy(list(z["prompt"]), len(z["tokens"]))
    assert toks == list(z["tokens"])
    np.testing.assert_allclose(lg, z["logits"], rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_head_bounds_contain_exact_logits(seed):
    """The property the greedy pick rests on (vocab8.py:1-12): every exact logit lies in [a - B, a + B], so the
    argmax row always has HI >= LO -- on random heads with rows of very different scales, an all-zero row,
    and tokens whose h has large and tiny entries."""
    g = np.random.default_rng(seed)
    V, D, T = 400, 128, 4
    w = (g.standard_normal((V, D)) * 0.02).astype(np.float32)
    w[::7] *= 300.0
    w[5] = 0.0
    wb = codec.f32_to_bf16_bits(w)
    h = g.standard_normal((T, D)).astype(np.float32)
    h[1, :8] *= 1e4
    h[2] *= 1e-3
    Q, S, C1, C2, AM = head.tables(wb)
    hi, lo = head.bounds(h, Q, S, C1, C2, AM)
    ex = head.exact_logits(wb, h)
    assert (ex <= hi).all()
    assert (ex.max(1) >= lo).all()
    for t in range(T):  # the argmax is always a candidate
        assert hi[t, int(np.argmax(ex[t]))] >= lo[t]
