"""Failures of the vocab-sharded exchange, made on the host over two gloo
ranks on CPU (no GPU is involved, none can hang):

- a truncated block: one rank sends [B][k-1] candidates; every rank raises
  ShardExchangeError naming it, and none goes on to the mismatched all-gather;
- a rank that leaves between steps (its process exits): the other rank's next
  collective ends with ShardExchangeError;
- a rank that stays but never joins the next collective: the process group's
  short timeout ends the other rank's collective with ShardExchangeError.
Each failing rank records what it saw in a file; the test checks the files.
"""
import datetime
import os
import socket
import time

import numpy as np
import pytest

from qwenium_b200 import shard


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, outdir, scenario):
    import torch
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=3))
    B, k, V = 4, 16, 1000
    lo, n = shard.shard_range(V, world, rank)
    outcome = "ok"
    t0 = time.monotonic()
    try:
        if scenario == "truncated":
            shard.check_layout(B, k - 1 if rank == 1 else k, lo, n, V)
        elif scenario in ("exits", "stalls"):
            shard.check_layout(B, k, lo, n, V)  # a first step every rank takes
            if rank == 1:
                if scenario == "stalls":
                    time.sleep(8)  # alive, but never joins the next collective
                outcome = "left"
            else:
                cv = torch.zeros((B, k), dtype=torch.float32)
                ci = torch.zeros((B, k), dtype=torch.int32)
                shard.exchange_candidates(cv, ci)
    except shard.ShardExchangeError as e:
        outcome = "error: " + str(e).replace("\n", " ")[:400]
    with open(os.path.join(outdir, f"rank{rank}.txt"), "w") as f:
        f.write(f"{time.monotonic() - t0:.2f}\n{outcome}\n")
    if scenario == "exits" and rank == 1:
        os._exit(0)  # leaves without tearing the group down
    try:
        dist.destroy_process_group()
    except Exception:
        pass
    os._exit(0)


def _run(tmp_path, scenario):
    import torch.multiprocessing as mp

    port = _port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, 2, port, str(tmp_path), scenario)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    out = {}
    for r in range(2):
        el, what = (tmp_path / f"rank{r}.txt").read_text().splitlines()[:2]
        out[r] = (float(el), what)
    return out


def test_truncated_block_is_rejected_on_every_rank(tmp_path):
    out = _run(tmp_path, "truncated")
    for r in range(2):
        assert out[r][1].startswith("error:"), out
        assert "rank 0 [4][16], rank 1 [4][15]" in out[r][1], out


@pytest.mark.parametrize("scenario", ["exits", "stalls"])
def test_missing_rank_ends_the_next_collective(tmp_path, scenario):
    out = _run(tmp_path, scenario)
    assert out[1][1] == "left", out
    el, what = out[0]
    assert what.startswith("error:") and "did not join" in what, out
    assert el < 30.0, out  # the group's 3 s timeout (or the closed connection) ends it
