"""Vocab-sharded token selection across ranks (a tensor-parallel output head).

Rank r holds the logits of a contiguous vocabulary slice ``[v_offset,
v_offset + V_local)`` for every row, as a column-parallel lm_head produces
them. One selection step is:

1. ``Context.shard_topk`` on every rank: the row transform (soft-cap, allow
   mask, repetition / frequency / presence penalties over global history ids,
   /T) and the local top-k as (value, global id) pairs, sorted by (value desc,
   id asc), padded with id -1;
2. one all-gather of the ``[B][k]`` value and id blocks (NCCL; 8 bytes per
   candidate);
3. ``Context.merge_topk`` on every rank: the global top-k of the union, then
   top-p, softmax and the draw exactly as the unsharded path
   (src/sampling/sampling.cpp:158-193). Every rank computes the same ids.

With ``0 < top_k`` the reference's top-p and softmax only see the top-k set
(sampling.cpp:168-190), so the merge is exact: sharded and unsharded runs
return identical tokens.

A row with a full-vocabulary top-p (``top_k == 0``, or k past what the merge
holds) depends on sequential float sums over its whole sorted vocabulary
(sampling.cpp:170-177), which no per-rank summary reproduces. Such rows are
transposed instead: one all-to-all moves each rank's slices of them so that
rank q holds rows q, q + N, ... whole; every rank samples its share with the
unsharded kernels, and one all-gather of the 32-byte row results gives every
rank every row. Identical to the unsharded path by construction; the
exchange is (N - 1) / N of each rank's slices of those rows.
"""
from __future__ import annotations

from typing import Optional, Tuple

import numpy as np

from .qsamp import ROW_PARAMS, ROW_RESULT

KMAX = 1024        # largest k the candidate exchange serves
MERGE_CAP = 5120   # candidates per row the merge holds (n_ranks * k)


def shard_range(V_total: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous split of V_total ids over `world` ranks: (v_offset, V_local).
    The first V_total % world ranks hold one id more."""
    if world < 1 or not (0 <= rank < world):
        raise ValueError(f"rank {rank} of world {world}: expected 0 <= rank < world")
    if V_total < world:
        raise ValueError(f"V_total={V_total}: expected >= world ({world})")
    base, extra = divmod(V_total, world)
    v_offset = rank * base + min(rank, extra)
    return v_offset, base + (1 if rank < extra else 0)


def candidates_per_row(params) -> int:
    """The candidate count k every rank sends: the largest top_k of the
    temperature rows (1 when every row is greedy)."""
    p = np.ascontiguousarray(params, ROW_PARAMS)
    ks = p["top_k"][p["temperature"] > 0]
    return int(max(1, ks.max())) if ks.size else 1


class ShardExchangeError(RuntimeError):
    """The candidate exchange failed: the ranks disagree on the batch layout
    (a truncated or misaligned block), or a collective did not complete (a
    rank that never joined: the process group's timeout ended it). Every rank
    that reaches the failing step raises it."""


def check_layout(B: int, k: int, v_offset: int, V_local: int, V_total: int, group=None) -> None:
    """One small all-gather of every rank's (B, k, v_offset, V_local): every
    rank checks that the blocks have one shape and that the slices tile
    [0, V_total) in rank order, and raises ShardExchangeError otherwise, so
    that no rank goes on to an all-gather whose sizes differ."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" else torch.device("cpu")
    mine = torch.tensor([B, k, v_offset, V_local], dtype=torch.int64, device=dev)
    alls = torch.empty((world, 4), dtype=torch.int64, device=dev)
    try:
        if dist.get_backend(group) == "nccl":
            dist.all_gather_into_tensor(alls, mine, group=group)
        else:
            dist.all_gather(list(alls.unbind(0)), mine, group=group)
    except Exception as e:  # (gloo / NCCL raise their own types; a timeout among them)
        raise ShardExchangeError(f"layout exchange failed (a rank did not join in time?): {e}") from e
    t = alls.cpu().tolist()
    bad = []
    if len({(b, kk) for b, kk, _, _ in t}) > 1:
        bad.append("the ranks send blocks of different shapes: " +
                   ", ".join(f"rank {r} [{b}][{kk}]" for r, (b, kk, _, _) in enumerate(t)))
    expect = 0
    for r, (_, _, off, n) in enumerate(t):
        if off != expect or n < 0:
            bad.append(f"rank {r} holds [{off}, {off + n}), expected to start at {expect}")
        expect = off + n
    if expect != V_total:
        bad.append(f"the slices end at {expect}, expected V_total={V_total}")
    if bad:
        raise ShardExchangeError("candidate blocks do not line up: " + "; ".join(bad))


def exchange_candidates(cand_vals, cand_ids, group=None):
    """All-gather each rank's [B][k] candidate blocks into [world][B][k]
    (rank-major, the layout qsamp_merge_topk reads). Works on any
    torch.distributed backend; NCCL uses one all_gather_into_tensor per array.
    A collective that fails or times out raises ShardExchangeError."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    out_v = torch.empty((world,) + tuple(cand_vals.shape), dtype=cand_vals.dtype, device=cand_vals.device)
    out_i = torch.empty((world,) + tuple(cand_ids.shape), dtype=cand_ids.dtype, device=cand_ids.device)
    try:
        if dist.get_backend(group) == "nccl":
            dist.all_gather_into_tensor(out_v, cand_vals.contiguous(), group=group)
            dist.all_gather_into_tensor(out_i, cand_ids.contiguous(), group=group)
        else:
            dist.all_gather(list(out_v.unbind(0)), cand_vals.contiguous(), group=group)
            dist.all_gather(list(out_i.unbind(0)), cand_ids.contiguous(), group=group)
    except Exception as e:
        raise ShardExchangeError(f"candidate all-gather failed (a rank did not join in time?): {e}") from e
    return out_v, out_i


def candidate_rows(params, V_total: int, world: int) -> np.ndarray:
    """The rows the candidate exchange serves exactly: greedy rows and rows
    with 0 < top_k < V_total whose k fits the merge (the rest are
    transposed)."""
    p = np.ascontiguousarray(params, ROW_PARAMS)
    k = p["top_k"].astype(np.int64)
    return (p["temperature"] <= 0) | ((k > 0) & (k < V_total) & (k <= min(KMAX, MERGE_CAP // world)))


def transpose_rows(local, rows, cols, group=None):
    """All-to-all of this rank's slices of rows `rows` (global row indices,
    the same list on every rank): full row j of the list goes to rank
    j % world. `local` is this rank's [B][cols[rank]] block (logits, or the
    allow-mask words of a slice that starts at a multiple of 32 ids); cols[q]
    is rank q's column count. Returns (this rank's row indices,
    [n_own][sum(cols)] on local's device, the ranks' columns side by side in
    rank order)."""
    import torch
    import torch.distributed as dist

    world, rank = dist.get_world_size(group), dist.get_rank(group)
    rows = np.asarray(rows, np.int64)
    mine = [j for j in range(len(rows)) if j % world == rank]
    dest = [[j for j in range(len(rows)) if j % world == q] for q in range(world)]
    order = np.concatenate([rows[d] for d in dest]).astype(np.int64)
    # moved as bytes (the collective needs no type of its own: bf16 bits,
    # mask words and fp32 logits alike)
    esz = local.element_size()
    bcols = [int(c) * esz for c in cols]
    send = local.index_select(0, torch.as_tensor(order, device=local.device)).contiguous().view(torch.uint8).view(-1)
    in_splits = [len(d) * bcols[rank] for d in dest]
    out_splits = [len(mine) * bcols[q] for q in range(world)]
    recv = torch.empty(sum(out_splits), dtype=torch.uint8, device=local.device)
    try:
        dist.all_to_all_single(recv, send, out_splits, in_splits, group=group)
    except Exception as e:
        raise ShardExchangeError(f"row all-to-all failed (a rank did not join in time?): {e}") from e
    full = torch.empty((len(mine), sum(bcols)), dtype=torch.uint8, device=local.device)
    off_r, off_c = 0, 0
    for q in range(world):
        n = len(mine) * bcols[q]
        full[:, off_c:off_c + bcols[q]] = recv[off_r:off_r + n].view(len(mine), bcols[q])
        off_r += n
        off_c += bcols[q]
    return rows[mine], full.view(local.dtype)


def gather_results(res_own, own_rows, B: int, out, group=None):
    """Every rank's [n_own][32] row results into out[B][32] on every rank."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    nmax = torch.tensor([len(own_rows)], dtype=torch.int64, device=res_own.device)
    dist.all_reduce(nmax, op=dist.ReduceOp.MAX, group=group)
    n = int(nmax.item())
    pad = torch.zeros((n, ROW_RESULT.itemsize), dtype=torch.uint8, device=res_own.device)
    pad[:len(own_rows)] = res_own
    ids = torch.full((n,), -1, dtype=torch.int64, device=res_own.device)
    ids[:len(own_rows)] = torch.as_tensor(own_rows, dtype=torch.int64, device=res_own.device)
    all_res = torch.empty((world, n, ROW_RESULT.itemsize), dtype=torch.uint8, device=res_own.device)
    all_ids = torch.empty((world, n), dtype=torch.int64, device=res_own.device)
    try:
        dist.all_gather(list(all_res.unbind(0)), pad, group=group)
        dist.all_gather(list(all_ids.unbind(0)), ids, group=group)
    except Exception as e:
        raise ShardExchangeError(f"result all-gather failed (a rank did not join in time?): {e}") from e
    keep = all_ids.view(-1) >= 0
    out[all_ids.view(-1)[keep]] = all_res.view(-1, ROW_RESULT.itemsize)[keep]
    return out


def sample_vshard(ctx, local_logits, params, V_total: int, hist=None, hist_len=None, masks=None,
                  u: Optional[np.ndarray] = None, rng_offset: int = 0, k: Optional[int] = None, group=None,
                  v_offset: Optional[int] = None, out_ids=None, out_results=None, comm=None,
                  check: bool = False):
    """One vocab-sharded selection step on this rank (steps 1-3 above).
    local_logits [B][V_local] is this rank's slice (by default the slice
    shard_range gives this rank). The exchange runs over `comm` (a
    qwenium_b200.comm.Comm: NCCL with deadlines; the call then waits for the
    step and raises CommError on a timeout or an aborted communicator) or
    else over torch.distributed; check=True first verifies that every rank's
    block lines up (check_layout). Rows with a full-vocabulary top-p take the
    transpose path (torch.distributed only; u required). Returns the row
    results (uint8 [B][32], ROW_RESULT layout), identical on every rank."""
    import torch

    if comm is not None:
        rank, world = comm.rank, comm.nranks
    else:
        import torch.distributed as dist

        rank, world = dist.get_rank(group), dist.get_world_size(group)
    B, V_local = int(local_logits.shape[0]), int(local_logits.shape[1])
    if v_offset is None:
        v_offset, V_expect = shard_range(V_total, world, rank)
        if V_expect != V_local:
            raise ValueError(f"local_logits has {V_local} columns; rank {rank} of {world} "
                             f"holds {V_expect} of V_total={V_total}")
    p = np.ascontiguousarray(params, ROW_PARAMS)
    cand = candidate_rows(p, V_total, world)
    if cand.all():
        kc = candidates_per_row(p) if k is None else int(k)
        if check and comm is None:
            check_layout(B, kc, v_offset, V_local, V_total, group)
        vals, ids = ctx.shard_topk(local_logits, p, v_offset, V_total, kc, hist=hist, hist_len=hist_len,
                                   masks=masks)
        if comm is not None:
            all_vals, all_ids = comm.allgather_candidates(vals, ids)
        else:
            all_vals, all_ids = exchange_candidates(vals, ids, group)
        res = ctx.merge_topk(all_vals, all_ids, p, u=u, rng_offset=rng_offset, out_ids=out_ids,
                             out_results=out_results)
        if comm is not None:
            comm.wait(device=local_logits.device)
        return res
    # rows with a full-vocabulary top-p: transposed (see the module docstring)
    if comm is not None:
        raise ShardExchangeError("rows with a full-vocabulary top-p are transposed with an all-to-all: "
                                 "use the torch.distributed exchange (comm=None)")
    if u is None:
        raise ValueError("u: rows with a full-vocabulary top-p need the per-row uniforms (the on-device "
                         "generator keys its draws by the row's place in the call)")
    u = np.ascontiguousarray(u, np.float64)
    hl = None if hist_len is None else np.ascontiguousarray(hist_len, np.int32)
    dev = local_logits.device
    out = out_results if out_results is not None else torch.empty((B, ROW_RESULT.itemsize), dtype=torch.uint8,
                                                                  device=dev)
    crow, frow = np.nonzero(cand)[0], np.nonzero(~cand)[0]
    if len(crow):
        ci = torch.as_tensor(crow, device=dev)
        pc = p[crow]
        kc = candidates_per_row(pc) if k is None else int(k)
        sub_h = hist.index_select(0, ci) if hist is not None else None
        sub_m = masks.index_select(0, ci) if masks is not None else None
        vals, ids = ctx.shard_topk(local_logits.index_select(0, ci), pc, v_offset, V_total, kc, hist=sub_h,
                                   hist_len=None if hl is None else hl[crow], masks=sub_m)
        all_vals, all_ids = exchange_candidates(vals, ids, group)
        out[ci] = ctx.merge_topk(all_vals, all_ids, pc, u=u[crow])
    spans = [shard_range(V_total, world, q) for q in range(world)]
    own, full = transpose_rows(local_logits, frow, [n for _, n in spans], group)
    fmask = None
    if masks is not None:
        if any(o % 32 for o, _ in spans):
            raise ShardExchangeError("allow-masks of full-vocabulary rows need every slice to start at a "
                                     "multiple of 32 ids")
        words = [n // 32 if q < world - 1 else (n + 31) // 32 for q, (_, n) in enumerate(spans)]
        _, fmask = transpose_rows(masks.view(torch.int32), frow, words, group)
    res_f = torch.empty((len(own), ROW_RESULT.itemsize), dtype=torch.uint8, device=dev)
    if len(own):
        oi = torch.as_tensor(own, device=dev)
        res_f = ctx.sample_batch(full, p[own], hist=hist.index_select(0, oi) if hist is not None else None,
                                 hist_len=None if hl is None else hl[own], masks=fmask, u=u[own])
    gather_results(res_f, own, B, out, group)
    if out_ids is not None:
        out_ids.copy_(out.view(torch.int32)[:, 0])
    return out
