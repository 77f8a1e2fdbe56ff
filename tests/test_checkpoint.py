"""HF checkpoint folder round trip: `save_checkpoint` writes config.json + model.safetensors (unfused tensors,
the names of the reference's loader, formats/model.py:37-106) and `Ckpt` reads them back into the fused
layer dict the engine consumes."""
import json
import os

import pytest
import torch

from ai_b200.model import CONFIGS, Ckpt, RandomWeights, layer_tensor_names, save_checkpoint


@pytest.mark.parametrize("name", ["tiny", "tiny-tied"])
def test_save_then_ckpt_reads_every_tensor(tmp_path, name):
    cfg = CONFIGS[name]
    rw = RandomWeights(cfg, seed=5, norm_noise=0.1)
    path = str(tmp_path / name)
    save_checkpoint(path, cfg, rw)
    ck = Ckpt(path)
    c = ck.config
    assert (c.L, c.D, c.H, c.KV, c.HD, c.FF, c.V, c.tied) == (cfg.L, cfg.D, cfg.H, cfg.KV, cfg.HD, cfg.FF, cfg.V,
                                                              cfg.tied)
    assert c.eps == cfg.eps and c.theta == cfg.theta
    for i in range(cfg.L):
        a, b = rw.layer(i), ck.layer(i)
        assert set(a) == set(b)
        for k in a:
            assert a[k].dtype == b[k].dtype and torch.equal(a[k], b[k]), (i, k)
        small = ck.layer_small(i)
        for k in small:
            assert torch.equal(small[k], a[k])
    assert torch.equal(ck.embedding(), rw.embedding())
    assert torch.equal(ck.final_norm(), rw.final_norm())
    assert torch.equal(ck.head(), rw.head())
    assert ck.head_name() == ("model.embed_tokens.weight" if cfg.tied else "lm_head.weight")
    # the unfused HF names are what is on disk (q/k/v and gate/up separately)
    names = layer_tensor_names(0)
    assert ck.mm(names["q"]).shape == (cfg.H * cfg.HD, cfg.D)
    assert ck.mm(names["gate"]).shape == (cfg.FF, cfg.D)


def test_ckpt_refuses_other_architectures(tmp_path):
    os.makedirs(tmp_path / "m")
    with open(tmp_path / "m" / "config.json", "w") as f:
        json.dump({"model_type": "llama"}, f)
    with pytest.raises(NotImplementedError):
        Ckpt(str(tmp_path / "m"))
    with pytest.raises(FileNotFoundError):
        Ckpt(str(tmp_path / "missing"))


@pytest.mark.gpu
def test_engine_from_saved_checkpoint_matches_in_memory_weights(tmp_path):
    """An Engine loaded from the saved folder (the HF path) decodes the same greedy tokens as one built from
    the same weights in memory."""
    from ai_b200.engine import Engine
    cfg = CONFIGS["tiny"]
    rw = RandomWeights(cfg, seed=7, norm_noise=0.1, std=0.05)
    path = str(tmp_path / "tiny")
    save_checkpoint(path, cfg, rw)
    a = Engine(cfg, maxt=64, weights=rw, log=None)
    b = Engine(path, maxt=64, log=None)
    prompt = [3, 1, 4, 1, 5, 9, 2, 6]
    assert list(a.generate(prompt, max_new=12)) == list(b.generate(prompt, max_new=12))
