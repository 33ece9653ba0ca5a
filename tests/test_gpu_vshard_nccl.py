"""Vocab-sharded selection over real ranks: 2 processes, one GPU each, NCCL.

Each rank holds its contiguous vocabulary slice; qwenium_b200.shard runs
shard_topk, the NCCL all-gather and merge_topk. Both ranks must return the
rows the unsharded path returns for the whole vocabulary. A second batch
mixes in rows with a full-vocabulary top-p (bf16, soft-cap, allow-masks),
which the shard path transposes with an NCCL all-to-all. Skipped with fewer
than two GPUs.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, outdir):
    import datetime

    import torch
    import torch.distributed as dist

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        from qwenium_b200 import qsamp, shard
        from test_gpu_vshard import RES, case, run_unsharded, to_dev

        ctx = qsamp.Context(rank)
        cfg = case(61, 64, 100003)
        base = run_unsharded(ctx, cfg)
        lo, n = shard.shard_range(cfg["logits"].shape[1], world, rank)
        local = to_dev(np.ascontiguousarray(cfg["logits"][:, lo:lo + n]), False)
        res = shard.sample_vshard(ctx, local, cfg["params"], cfg["logits"].shape[1],
                                  hist=torch.from_numpy(cfg["hist"]).cuda(), hist_len=cfg["hist_len"], u=cfg["u"])
        torch.cuda.synchronize()
        got = res.cpu().numpy().view(RES).reshape(-1)
        np.save(os.path.join(outdir, f"got{rank}.npy"), got)
        np.save(os.path.join(outdir, f"base{rank}.npy"), base)
        # rows with a full-vocabulary top-p among candidate rows
        from test_gpu_vshard import slice_mask

        cfg2 = case(64, 48, 131072, bf16=True, masks=True)
        p2 = cfg2["params"]
        p2["top_k"][::3] = 0
        p2["temperature"][::3] = 0.9
        V2 = cfg2["logits"].shape[1]
        base2 = run_unsharded(ctx, cfg2)
        lo, n = shard.shard_range(V2, world, rank)
        local2 = to_dev(np.ascontiguousarray(cfg2["logits"][:, lo:lo + n]), True)
        lmask = torch.from_numpy(np.ascontiguousarray(slice_mask(cfg2["masks"], lo, n)).view(np.int32)).cuda()
        res2 = shard.sample_vshard(ctx, local2, p2, V2, hist=torch.from_numpy(cfg2["hist"]).cuda(),
                                   hist_len=cfg2["hist_len"], masks=lmask, u=cfg2["u"])
        torch.cuda.synchronize()
        np.save(os.path.join(outdir, f"got2_{rank}.npy"), res2.cpu().numpy().view(RES).reshape(-1))
        np.save(os.path.join(outdir, f"base2_{rank}.npy"), base2)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_vshard_two_ranks_nccl(tmp_path):
    import torch
    import torch.multiprocessing as mp

    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
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
        got = np.load(tmp_path / f"got{r}.npy")
        base = np.load(tmp_path / f"base{r}.npy")
        assert_same(got, base, f"rank {r}")
        assert_same(np.load(tmp_path / f"got2_{r}.npy"), np.load(tmp_path / f"base2_{r}.npy"),
                    f"rank {r}, full-vocabulary rows transposed")
