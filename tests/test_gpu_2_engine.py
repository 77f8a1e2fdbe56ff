"""Whole-model parity: the engine's greedy tokens equal the CPU oracle's on random-init Qwen3 models."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def oracle_for(cfg, rw, maxt):
    """The oracle decode with the reference head's arithmetic (exact_rows: fp32 products, sequential sum)."""
    from oracle.model import DecodeOracle
    layers = [{k: bits(v) for k, v in rw.layer(i).items()} for i in range(cfg.L)]
    return DecodeOracle(cfg, layers, bits(rw.embedding()), bits(rw.head()), bits(rw.final_norm()), maxt,
                        exact_head=True)


@pytest.fixture(scope="module", params=["tiny", "tiny-tied", "small", "small-1k"])
def pair(request, cuda_dev):
    from ai_b200 import build
    from ai_b200.engine import Engine
    from ai_b200.model import CONFIGS, RandomWeights
    build.build()
    cfg = CONFIGS[request.param]
    rw = RandomWeights(cfg, seed=11, norm_noise=0.1, std=0.05)
    eng = Engine(cfg, maxt=128, weights=rw, log=None)
    return cfg, rw, eng


def test_greedy_generate_matches_oracle(pair):
    cfg, rw, eng = pair
    prompt = [int(t) for t in np.random.default_rng(1).integers(0, cfg.V, 20)]
    toks = list(eng.generate(prompt, max_new=24))
    o = oracle_for(cfg, rw, 128)
    ref, lg = o.greedy(prompt, 24)
    assert toks == ref
    from ai_b200._lib import status
    assert status() == 0


def test_process_rows_match_oracle_logit_argmax(pair):
    cfg, rw, eng = pair
    toks = [int(t) for t in np.random.default_rng(2).integers(0, cfg.V, 9)]
    out = eng.process(toks, 0)
    o = oracle_for(cfg, rw, 128)
    ref = []
    for p, t in enumerate(toks):
        lg = o.step(t, p)
        ref.append(int(np.flatnonzero(lg == lg.max()).min()))
    assert out == ref
    # continue with a single token at position 9 through the T=1 graph
    assert eng.process([toks[-1]], 9) == [int(np.argmax(o.step(toks[-1], 9)))]


def test_sampling_reproducible_and_graph_equals_eager(pair):
    cfg, rw, eng = pair
    prompt = [3, 1, 4, 1, 5]
    a = list(eng.generate(prompt, max_new=12, temperature=0.8, top_p=0.9, top_k=20, seed=7))
    b = list(eng.generate(prompt, max_new=12, temperature=0.8, top_p=0.9, top_k=20, seed=7))
    assert a == b
    eng.use_graphs = False
    c = list(eng.generate(prompt, max_new=12, temperature=0.8, top_p=0.9, top_k=20, seed=7))
    eng.use_graphs = True
    assert a == c


def test_sampled_steps_match_head_pick(pair):
    """Sampling at temperature > 0 picks, at every decode step, the token the reference's Head.pick draws for the
    same hidden state and the same uniform: exact fp32 logits of the whole vocabulary (exact_rows, head.py:19-26 --
    here recomputed by the oracle from the engine's own final-norm output) and the sampler's steps with the
    step's draw from np.random.default_rng(seed). (Whole trajectories are compared with greedy decoding: a sampled
    trajectory depends on hidden-state rounding wherever a draw lands within ~1e-7 of a CDF boundary.)"""
    from oracle import head as ohead, sampler as osamp
    cfg, rw, eng = pair
    head_bits = bits(rw.head())
    prompt = [int(t) for t in np.random.default_rng(5).integers(0, cfg.V, 7)]
    for seed, (temp, k, p) in [(3, (0.6, 20, 0.8)), (4, (1.0, 0, 0.95)), (5, (0.7, 1, 1.0))]:
        rng = np.random.default_rng(seed)
        gen = eng.generate(prompt, max_new=16, temperature=temp, top_k=k, top_p=p, seed=seed)
        next(gen)
        rng.random()  # the prompt pass's draw
        n = 0
        for tok in gen:
            h = eng.hb[0].cpu().numpy()[None]
            lg = ohead.exact_logits(head_bits, h)[0]
            assert tok == osamp.sample_row(lg, temp, k, p, u=rng.random()), (seed, n)
            n += 1
        assert n == 15


def test_penalties_change_greedy_path(pair):
    cfg, rw, eng = pair
    prompt = [7, 7, 7, 7]
    plain = list(eng.generate(prompt, max_new=8))
    pen = list(eng.generate(prompt, max_new=8, repetition_penalty=50.0, presence_penalty=5.0))
    assert 7 not in pen[:1] or pen != plain


def test_process_errors_like_reference(pair):
    cfg, rw, eng = pair
    with pytest.raises(ValueError):
        eng.process([], 0)
    with pytest.raises(ValueError):
        eng.process([cfg.V], 0)
    with pytest.raises(ValueError):
        eng.process([1], 10 ** 6)


def test_codec_cache_reload(tmp_path):
    """An engine loaded from the on-disk codec file (written by a first load) holds the same planes and
    decodes the same greedy tokens; a file made for other weights is refused."""
    from ai_b200.engine import Engine
    from ai_b200.model import CONFIGS, RandomWeights
    cfg = CONFIGS["small-1k"]
    rw = RandomWeights(cfg, seed=11, norm_noise=0.1, std=0.05)
    path = str(tmp_path / "small-1k.codec")
    a = Engine(cfg, maxt=64, weights=rw, log=None, codec_cache=path)
    b = Engine(cfg, maxt=64, weights=rw, log=None, codec_cache=path)
    for la, lb in zip(a.W, b.W):
        for n in la:
            for k in ("m8", "e4", "rp", "ec", "ev"):
                assert torch.equal(la[n][k], lb[n][k])
    prompt = [5, 4, 3, 2, 1]
    assert list(a.generate(prompt, max_new=8)) == list(b.generate(prompt, max_new=8))
    with pytest.raises(ValueError):
        Engine(cfg, maxt=64, weights=RandomWeights(cfg, seed=12, norm_noise=0.1, std=0.05), log=None,
               codec_cache=path)


def test_speculative_greedy_equals_plain():
    """Greedy decoding verified against a draft engine gives the plain greedy tokens: with the same model as
    drafter every proposal is accepted, with another model most are rejected and corrected."""
    from ai_b200.engine import Engine
    from ai_b200.model import CONFIGS, RandomWeights
    cfg = CONFIGS["small"]
    tgt = Engine(cfg, maxt=128, weights=RandomWeights(cfg, seed=11, norm_noise=0.1, std=0.05), log=None)
    same = Engine(cfg, maxt=128, weights=RandomWeights(cfg, seed=11, norm_noise=0.1, std=0.05), log=None)
    other = Engine(cfg, maxt=128, weights=RandomWeights(cfg, seed=29, norm_noise=0.1, std=0.05), log=None)
    prompt = [int(t) for t in np.random.default_rng(4).integers(0, cfg.V, 12)]
    plain = list(tgt.generate(prompt, max_new=40))
    st1, st2 = {}, {}
    assert list(tgt.generate(prompt, max_new=40, draft=same, k=7, stats=st1)) == plain
    assert st1["accepted"] == st1["drafted"] and st1["passes"] < 39
    assert list(tgt.generate(prompt, max_new=40, draft=other, stats=st2)) == plain
    assert st2["accepted"] < st2["drafted"]
    with pytest.raises(NotImplementedError):
        list(tgt.generate(prompt, max_new=4, draft=same, temperature=0.7))


def test_batch_decode_equals_single_sequences(pair):
    """Sequences decoded together (one weight read per step for all of them, each attending its own cache at its
    own position) give each sequence's own greedy tokens."""
    cfg, rw, eng = pair
    g = np.random.default_rng(12)
    prompts = [[int(t) for t in g.integers(0, cfg.V, n)] for n in (5, 20, 33)]
    alone = [list(eng.generate(p, max_new=10)) for p in prompts]
    assert eng.generate_batch(prompts, max_new=10) == alone
    from ai_b200._lib import status
    assert status() == 0
