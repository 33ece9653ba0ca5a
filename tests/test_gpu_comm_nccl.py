"""The native candidate exchange (libqsamp_comm.so) on two GPUs: two
processes, one GPU each, a non-blocking NCCL communicator with a 3 s
deadline, no torch.distributed.

Step 1: vocab-sharded selection with the exchange over the communicator; both
ranks must return the rows the unsharded path returns.
Step 2: rank 1 stops between steps -- alive, nothing of it in flight, but it
never joins the next all-gather (NVLS off); rank 0's next step cannot
complete and must end with TIMEOUT (or COMM) at its deadline, its
communicator must report itself aborted, and the GPU must still serve an
unsharded call with the same rows. Rank 1 then destroys its communicator and
exits.
Skipped with fewer than two GPUs.
"""
import os
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _worker(rank, world, outdir):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ.setdefault("NCCL_DEBUG", "WARN")
    import torch

    torch.cuda.set_device(rank)
    from qwenium_b200 import comm, qsamp, shard
    from test_gpu_vshard import RES, case, run_unsharded, to_dev

    idfile = os.path.join(outdir, "uid.bin")
    if rank == 0:
        with open(idfile + ".tmp", "wb") as f:
            f.write(comm.unique_id())
        os.replace(idfile + ".tmp", idfile)
    t0 = time.monotonic()
    while not os.path.exists(idfile):
        if time.monotonic() - t0 > 60:
            raise RuntimeError("no communicator id")
        time.sleep(0.05)
    uid = open(idfile, "rb").read()
    c = comm.Comm(world, rank, uid, rank, timeout_ms=3000)
    ctx = qsamp.Context(rank)
    cfg = case(63, 64, 100003)
    V = cfg["logits"].shape[1]
    base = run_unsharded(ctx, cfg)
    lo, n = shard.shard_range(V, world, rank)
    local = to_dev(np.ascontiguousarray(cfg["logits"][:, lo:lo + n]), False)
    hist = torch.from_numpy(cfg["hist"]).cuda()
    res = shard.sample_vshard(ctx, local, cfg["params"], V, hist=hist, hist_len=cfg["hist_len"], u=cfg["u"],
                              comm=c)
    got = res.cpu().numpy().view(RES).reshape(-1)
    np.save(os.path.join(outdir, f"got{rank}.npy"), got)
    np.save(os.path.join(outdir, f"base{rank}.npy"), base)
    if rank == 1:
        # stops between steps: nothing of this rank is in flight, and it does
        # not join rank 0's next all-gather
        with open(os.path.join(outdir, "stopped1"), "w") as f:
            f.write("stopped")
        t0 = time.monotonic()
        while not os.path.exists(os.path.join(outdir, "done0")) and time.monotonic() - t0 < 90:
            time.sleep(0.05)
        c.close()
        os._exit(0)
    # rank 0: the next step, without rank 1
    t0 = time.monotonic()
    while not os.path.exists(os.path.join(outdir, "stopped1")) and time.monotonic() - t0 < 60:
        time.sleep(0.05)
    t0 = time.monotonic()
    outcome = "completed"
    try:
        r2 = shard.sample_vshard(ctx, local, cfg["params"], V, hist=hist, hist_len=cfg["hist_len"], u=cfg["u"],
                                 comm=c)
        g2 = r2.cpu().numpy().view(RES).reshape(-1)
        outcome = f"completed (rows equal to the unsharded ones: {bool(np.array_equal(g2, base))})"
    except comm.CommError as e:
        outcome = f"{comm.STATUS.get(e.status)} {e}"
    el = time.monotonic() - t0
    alive = c.alive()
    c.close()
    again = run_unsharded(ctx, cfg)  # the context and the GPU still serve
    np.save(os.path.join(outdir, "again0.npy"), again)
    with open(os.path.join(outdir, "step2.txt"), "w") as f:
        f.write(f"{el:.2f}\n{int(alive)}\n{outcome}\n")
    with open(os.path.join(outdir, "done0"), "w") as f:
        f.write("done")
    os._exit(0)


def test_native_exchange_and_a_rank_that_stops(tmp_path):
    import torch
    import torch.multiprocessing as mp

    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, 2, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    from test_gpu_vshard import assert_same

    for r in range(2):
        assert_same(np.load(tmp_path / f"got{r}.npy"), np.load(tmp_path / f"base{r}.npy"), f"rank {r}")
    el, alive, outcome = (tmp_path / "step2.txt").read_text().splitlines()[:3]
    assert outcome.startswith("TIMEOUT") or outcome.startswith("COMM"), outcome
    assert float(el) < 30.0 and alive == "0", (el, alive, outcome)
    assert_same(np.load(tmp_path / "again0.npy"), np.load(tmp_path / "base0.npy"), "rank 0 after the abort")
