"""Host logic of the vocab-sharded path on CPU: the vocabulary split, the
candidate count, and the all-gather layout that qsamp_merge_topk reads, over
two gloo ranks. The per-rank top-k and the merge are computed here by a
plain numpy restatement (the kernels need a GPU); the check is that merging
the exchanged candidates gives the unsharded top-k, ids and order."""
import os
import socket

import numpy as np
import pytest

from qwenium_b200 import shard
from qwenium_b200 import workloads as W


def test_shard_range_covers_vocab():
    for V in (1, 7, 32, 151936, 262144, 100003):
        for world in (1, 2, 3, 8):
            if V < world:
                with pytest.raises(ValueError):
                    shard.shard_range(V, world, 0)
                continue
            spans = [shard.shard_range(V, world, r) for r in range(world)]
            assert spans[0][0] == 0
            for (o1, n1), (o2, _) in zip(spans, spans[1:]):
                assert o1 + n1 == o2
            assert spans[-1][0] + spans[-1][1] == V
            assert max(n for _, n in spans) - min(n for _, n in spans) <= 1
    with pytest.raises(ValueError):
        shard.shard_range(10, 2, 2)


def test_candidates_per_row():
    p = W.default_params(4)
    p["top_k"] = [5, 64, 0, 3]
    p["temperature"] = [1.0, 0.0, 1.0, 1.0]  # the greedy row's k does not count
    assert shard.candidates_per_row(p) == 5
    p["temperature"] = 0.0
    assert shard.candidates_per_row(p) == 1


def _topk(vals, ids, k):
    # (value desc, id asc)
    order = np.lexsort((ids, -vals.astype(np.float64)))
    return vals[order][:k], ids[order][:k]


def _worker(rank, world, port, outdir):
    import datetime

    import torch
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        B, V, k = 6, 1003, 16
        rng = np.random.default_rng(7)
        x = (rng.standard_normal((B, V)) * 3).astype(np.float32)
        x[:, 500:520] = np.float32(9.0)  # ties across the shard boundary
        lo, n = shard.shard_range(V, world, rank)
        cv = np.full((B, k), -np.inf, np.float32)
        ci = np.full((B, k), -1, np.int32)
        for b in range(B):
            v, i = _topk(x[b, lo:lo + n], np.arange(lo, lo + n, dtype=np.int32), k)
            cv[b, :len(v)], ci[b, :len(i)] = v, i
        av, ai = shard.exchange_candidates(torch.from_numpy(cv), torch.from_numpy(ci))
        np.save(os.path.join(outdir, f"v{rank}.npy"), av.numpy())
        np.save(os.path.join(outdir, f"i{rank}.npy"), ai.numpy())
        np.save(os.path.join(outdir, "x.npy"), x)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_exchange_layout_two_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    x = np.load(tmp_path / "x.npy")
    B, V = x.shape
    k = 16
    v0, i0 = np.load(tmp_path / "v0.npy"), np.load(tmp_path / "i0.npy")
    v1, i1 = np.load(tmp_path / "v1.npy"), np.load(tmp_path / "i1.npy")
    assert v0.shape == (2, B, k) and np.array_equal(v0, v1) and np.array_equal(i0, i1)  # same on every rank
    for r in range(2):  # rank-major: block r is rank r's ids
        lo, n = shard.shard_range(V, 2, r)
        ids = i0[r][i0[r] >= 0]
        assert np.all((ids >= lo) & (ids < lo + n))
    for b in range(B):
        vals, ids = v0[:, b, :].ravel(), i0[:, b, :].ravel()
        keep = ids >= 0
        mv, mi = _topk(vals[keep], ids[keep], k)
        ev, ei = _topk(x[b], np.arange(V, dtype=np.int32), k)
        assert np.array_equal(mi, ei) and np.array_equal(mv, ev)


def _transpose_worker(rank, world, port, outdir):
    import datetime

    import torch
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        B, V = 7, 2048
        rng = np.random.default_rng(5)
        x = rng.standard_normal((B, V)).astype(np.float32)
        bits = (rng.random((B, V)) < 0.5).astype(np.uint8)
        words = np.packbits(bits, axis=1, bitorder="little").view(np.int32).reshape(B, V // 32)
        lo, n = shard.shard_range(V, world, rank)
        rows = [1, 3, 4, 6]
        cols = [shard.shard_range(V, world, q)[1] for q in range(world)]
        own, full = shard.transpose_rows(torch.from_numpy(np.ascontiguousarray(x[:, lo:lo + n])), rows, cols)
        _, fmask = shard.transpose_rows(torch.from_numpy(np.ascontiguousarray(words[:, lo // 32:(lo + n) // 32])),
                                        rows, [c // 32 for c in cols])
        np.save(os.path.join(outdir, f"own{rank}.npy"), own)
        np.save(os.path.join(outdir, f"full{rank}.npy"), full.numpy())
        np.save(os.path.join(outdir, f"mask{rank}.npy"), fmask.numpy())
        # results: row r's record holds r in every byte
        res = torch.tensor(np.repeat(own.astype(np.uint8)[:, None], 32, axis=1))
        out = torch.zeros((B, 32), dtype=torch.uint8)
        shard.gather_results(res, own, B, out)
        np.save(os.path.join(outdir, f"out{rank}.npy"), out.numpy())
        np.save(os.path.join(outdir, "x.npy"), x)
        np.save(os.path.join(outdir, "words.npy"), words)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_full_vocabulary_rows_transpose_two_gloo_ranks(tmp_path):
    """Rows with a full-vocabulary top-p are moved whole to one rank each
    (row j of the list to rank j % 2) with their allow-mask words, and the
    row results come back to every rank."""
    import torch.multiprocessing as mp

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_transpose_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    x, words = np.load(tmp_path / "x.npy"), np.load(tmp_path / "words.npy")
    rows = [1, 3, 4, 6]
    for r in range(2):
        own = np.load(tmp_path / f"own{r}.npy")
        assert list(own) == rows[r::2]
        assert np.array_equal(np.load(tmp_path / f"full{r}.npy"), x[own])
        assert np.array_equal(np.load(tmp_path / f"mask{r}.npy"), words[own])
        out = np.load(tmp_path / f"out{r}.npy")
        for b in range(x.shape[0]):
            assert np.all(out[b] == (b if b in rows else 0)), (r, b, out[b])
