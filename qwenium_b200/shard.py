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
return identical tokens. A full-vocabulary top-p (``top_k == 0``) is not
served in this mode (the library answers UNSUPPORTED).
"""
from __future__ import annotations

from typing import Optional, Tuple

import numpy as np

from .qsamp import ROW_PARAMS


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
    block lines up (check_layout). Returns the row results (uint8 [B][32],
    ROW_RESULT layout), identical on every rank."""
    if comm is not None:
        rank, world = comm.rank, comm.nranks
    else:
        import torch.distributed as dist

        rank, world = dist.get_rank(group), dist.get_world_size(group)
    V_local = int(local_logits.shape[1])
    if v_offset is None:
        v_offset, V_expect = shard_range(V_total, world, rank)
        if V_expect != V_local:
            raise ValueError(f"local_logits has {V_local} columns; rank {rank} of {world} "
                             f"holds {V_expect} of V_total={V_total}")
    kc = candidates_per_row(params) if k is None else int(k)
    if check and comm is None:
        check_layout(int(local_logits.shape[0]), kc, v_offset, V_local, V_total, group)
    vals, ids = ctx.shard_topk(local_logits, params, v_offset, V_total, kc, hist=hist, hist_len=hist_len,
                               masks=masks)
    if comm is not None:
        all_vals, all_ids = comm.allgather_candidates(vals, ids)
    else:
        all_vals, all_ids = exchange_candidates(vals, ids, group)
    res = ctx.merge_topk(all_vals, all_ids, params, u=u, rng_offset=rng_offset, out_ids=out_ids,
                         out_results=out_results)
    if comm is not None:
        comm.wait(device=local_logits.device)
    return res
