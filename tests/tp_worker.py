"""One rank of the 2-GPU tensor-parallel check (launched by tests/test_gpu_3_tp.py through torchrun): every
rank runs the same greedy and sampled generations with Engine(tp=world); rank 0 also runs the single-GPU
engine on the same weights. Rank 0 prints one JSON line with every rank's tokens."""
import datetime
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def ar_check(eng, rank, world):
    """The one-shot all-reduce gives bitwise the rank-order sum of every rank's block, call after call (the
    epochs alternate the two buffer slots)."""
    if eng.ar is None:
        return None
    ok = True
    for i, n in enumerate((4096, 1000, eng.ar["nmax"], 4096)):
        g = torch.Generator(device="cuda").manual_seed(100 * i + rank)
        x = torch.randn(n, generator=g, device="cuda")
        parts = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(parts, x)
        want = torch.zeros_like(x)
        for p in parts:
            want += p
        eng._reduce(x)
        torch.cuda.synchronize()
        ok = ok and torch.equal(x, want)
    return ok


def main():
    rank, world, lr = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(lr)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60))
    from ai_b200 import build
    from ai_b200.engine import Engine
    from ai_b200.model import CONFIGS, RandomWeights
    build.build()
    cfg = CONFIGS[sys.argv[1]]
    rw = RandomWeights(cfg, seed=11, norm_noise=0.1, std=0.05)
    prompt = [3, 1, 4, 1, 5, 9, 2, 6, 5, 3, 5, 8, 9, 7, 9, 3, 2, 3, 8, 4]  # > 16 tokens: the batched path too
    eng = Engine(cfg, maxt=128, weights=rw, log=None, tp=world)
    res = {"oneshot": eng.ar is not None, "ar_exact": ar_check(eng, rank, world),
           "greedy": list(eng.generate(prompt, max_new=16)),
           "sample": list(eng.generate(prompt, max_new=12, temperature=0.8, top_p=0.9, top_k=20, seed=7))}
    eng.use_graphs = False
    res["eager"] = list(eng.generate(prompt, max_new=16))
    eng.close()
    if rank == 0:
        ref = Engine(cfg, maxt=128, weights=rw, log=None)
        res["ref_greedy"] = list(ref.generate(prompt, max_new=16))
        ref.close()
    from ai_b200._lib import status
    res["status"] = status()
    allres = [None] * world
    dist.all_gather_object(allres, res)
    if rank == 0:
        print(json.dumps(allres))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
