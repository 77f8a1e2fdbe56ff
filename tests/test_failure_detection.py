"""Host-side failure detection of the multi-rank path on CPU (gloo): a rank that never reaches a collective makes
the other rank's collective end with an error after the process group's timeout, instead of waiting forever."""
import datetime
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _rank(rank, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=3))
    if rank == 1:  # never joins the all-reduce
        time.sleep(12)
        return
    t0 = time.time()
    try:
        dist.all_reduce(torch.ones(4))
        out.put(("no error", time.time() - t0))
    except Exception as exc:  # noqa: BLE001 -- any error ends the wait, which is the property under test
        out.put((type(exc).__name__, time.time() - t0))


@pytest.mark.timeout(120)
def test_missing_rank_times_out_with_an_error():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    kind, waited = q.get(timeout=60)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert kind != "no error"
    assert waited < 11  # ended by the 3 s timeout, not by the peer's eventual exit
