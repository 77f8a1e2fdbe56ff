"""Tensor-parallel split of the decode layer, on the CPU: `model.shard_layer` and the residual convention the
engine uses (rank 0 adds its partial into x, the other ranks write theirs, one all-reduce sums them), checked
against the unsharded layer with two `gloo` ranks."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ai_b200.model import CONFIGS, RandomWeights, check_tp, shard_layer


def _full_update(lw, cfg, x, att):
    """o_proj residual update, then the SiLU-gated MLP update (RMSNorm weight ln2), in float64."""
    f = lambda t: t.double()  # noqa: E731
    x = x + f(lw["o"]) @ att
    h = x / torch.sqrt((x * x).mean() + cfg.eps) * f(lw["ln2"])
    g, u = torch.split(f(lw["gu"]), [cfg.FF, cfg.FF])
    mid = torch.nn.functional.silu(g @ h) * (u @ h)
    return x + f(lw["down"]) @ mid


def _rank_update(sh, cfg, x, att_r, rank, reduce):
    """The engine's order on one rank: partial o_proj (added into x on rank 0 only), all-reduce, norm of the
    reduced x, the rank's gate/up rows, partial down_proj (same convention), all-reduce."""
    f = lambda t: t.double()  # noqa: E731
    y = (x.clone() if rank == 0 else torch.zeros_like(x)) + f(sh["o"]) @ att_r
    x = reduce(y)
    h = x / torch.sqrt((x * x).mean() + cfg.eps) * f(sh["ln2"])
    fr = sh["gu"].shape[0] // 2
    g, u = torch.split(f(sh["gu"]), [fr, fr])
    mid = torch.nn.functional.silu(g @ h) * (u @ h)
    y = (x.clone() if rank == 0 else torch.zeros_like(x)) + f(sh["down"]) @ mid
    return reduce(y)


@pytest.mark.parametrize("name,n", [("tiny", 2), ("small", 2), ("small-1k", 2), ("small-1k", 4)])
def test_shards_reassemble(name, n):
    cfg = CONFIGS[name]
    lw = RandomWeights(cfg, seed=3, device="cpu").layer(0)
    shards = [shard_layer(lw, cfg, r, n) for r in range(n)]
    H, KV, HD, FF = cfg.H, cfg.KV, cfg.HD, cfg.FF
    q, k, v = torch.split(lw["qkv"], [H * HD, KV * HD, KV * HD])
    parts = [torch.split(s["qkv"], [H // n * HD, KV // n * HD, KV // n * HD]) for s in shards]
    assert torch.equal(torch.cat([p[0] for p in parts]), q)
    assert torch.equal(torch.cat([p[1] for p in parts]), k)
    assert torch.equal(torch.cat([p[2] for p in parts]), v)
    assert torch.equal(torch.cat([s["o"] for s in shards], 1), lw["o"])
    assert torch.equal(torch.cat([s["down"] for s in shards], 1), lw["down"])
    gs = [torch.split(s["gu"], [FF // n, FF // n]) for s in shards]
    assert torch.equal(torch.cat([g for g, _ in gs] + [u for _, u in gs]), lw["gu"])
    # the query heads of a rank use exactly its KV groups (GQA group = head // (H / KV))
    G = H // KV
    for r in range(n):
        heads = range(r * H // n, (r + 1) * H // n)
        assert {h // G for h in heads} == set(range(r * KV // n, (r + 1) * KV // n))


def test_split_rejected():
    with pytest.raises(ValueError):
        check_tp(CONFIGS["tiny"], 4)  # KV = 2
    with pytest.raises(ValueError):
        check_tp(CONFIGS["small"], 4)  # FF / 4 = 384 is not a multiple of 256


def _worker(rank, world, port, name):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = CONFIGS[name]
        lw = RandomWeights(cfg, seed=5, device="cpu").layer(1)
        g = torch.Generator().manual_seed(7)
        x = torch.randn(cfg.D, generator=g, dtype=torch.float64)
        att = torch.randn(cfg.H * cfg.HD, generator=g, dtype=torch.float64)
        hq = cfg.H // world * cfg.HD

        def reduce(t):
            dist.all_reduce(t)
            return t

        sh = shard_layer(lw, cfg, rank, world)
        got = _rank_update(sh, cfg, x, att[rank * hq:(rank + 1) * hq], rank, reduce)
        want = _full_update(lw, cfg, x, att)
        torch.testing.assert_close(got, want, rtol=1e-10, atol=1e-10)
        # every rank holds the same reduced state
        mx = got.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        assert torch.equal(mx, got)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("name", ["tiny", "small-1k"])
def test_two_rank_layer_update_matches_unsharded(name):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.spawn(_worker, args=(2, port, name), nprocs=2, join=True)
