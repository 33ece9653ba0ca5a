"""Failure detection on the GPU without a GPU fault.

Every wait in the kernels is bounded; when a bound runs out the kernel gives
the row up (token -1), sets the device status word and goes on, so the
context stays usable. The failures are made on the host:

* a row chunk whose arrival flag the host never raises
  (qsamp_limits.drop_ready_from) makes the kernels' ready waits run out;
* a gather-round budget of one (qsamp_limits.max_rounds) makes the
  full-vocabulary rows that need a second round give up.

Both surface as QSAMP_ERR_DEVICE: from qsamp_sample_host directly, and from
qsamp_poll_status after an asynchronous qsamp_sample. Rows not concerned
match the oracle bit for bit.
"""
import numpy as np
import pytest

import oracle as O
from qwenium_b200 import workloads as W

pytestmark = pytest.mark.gpu

FIELDS = ("token", "position", "n_keep", "drew", "sum_exp", "sum_keep", "max_logit", "prob")


@pytest.fixture()
def ctx():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from qwenium_b200 import qsamp

    c = qsamp.Context(0)
    yield c
    c.close()


def _same_rows(got, want, rows):
    bad = []
    for b in rows:
        for f in FIELDS:
            g, w = got[b][f], want[b][f]
            ok = (int(g) == int(w)) if f in FIELDS[:4] else (np.float32(g).view(np.uint32) == np.float32(w).view(np.uint32))
            if not ok:
                bad.append((b, f, g, w))
    return bad


def test_ready_wait_runs_out(ctx):
    from qwenium_b200 import qsamp

    cfg = W.config2(31, B=64)  # 64 x 608 KB: the host entry copies 6 row chunks of 11 rows
    want, _, _, _ = O.oracle_sample(cfg["logits"], cfg["params"], cfg["hist"], cfg["hist_len"], None, cfg["u"])
    ctx.set_limits(ready_wait_ns=2_000_000, drop_ready_from=3)
    st = []
    _, got, _, _ = ctx.sample_host(cfg["logits"], cfg["params"], cfg["hist"], cfg["hist_len"], None, cfg["u"],
                                   status_out=st)
    assert st and st[0][0] == 4 and "bounded wait" in st[0][1], st
    chunk = (64 + 5) // 6
    lost = np.arange(64) >= 3 * chunk
    assert np.all(got["token"][lost] == -1) and np.all(got["position"][lost] == -1)
    assert not _same_rows(got, want, np.nonzero(~lost)[0])
    # the context stays usable: every flag raised again, every row served
    ctx.set_limits(ready_wait_ns=1_000_000_000, drop_ready_from=-1)
    _, got2, _, _ = ctx.sample_host(cfg["logits"], cfg["params"], cfg["hist"], cfg["hist_len"], None, cfg["u"])
    assert not _same_rows(got2, want, range(64))
    with pytest.raises(qsamp.QsampError):
        ctx.set_limits(max_rounds=0)


def test_round_budget_runs_out(ctx):
    import torch

    from qwenium_b200 import qsamp

    cfg = W.config2(2000, B=256)
    want, _, _, _ = O.oracle_sample(cfg["logits"], cfg["params"], cfg["hist"], cfg["hist_len"], None, cfg["u"])
    x = torch.from_numpy(cfg["logits"]).cuda()
    hist = torch.from_numpy(cfg["hist"]).cuda()
    ids = torch.empty(256, dtype=torch.int32, device="cuda")

    def run():
        res = ctx.sample_batch(x, cfg["params"], hist=hist, hist_len=cfg["hist_len"], u=cfg["u"], out_ids=ids)
        torch.cuda.synchronize()
        return res.cpu().numpy().view(qsamp.ROW_RESULT).reshape(-1)

    ctx.set_limits(max_rounds=1)
    got = run()
    failed = got["token"] == -1
    assert failed.any(), "no row of this batch needed a second gather round"
    with pytest.raises(qsamp.QsampError) as ei:
        ctx.poll_status()
    assert ei.value.status == 4 and "gather rounds" in str(ei.value)
    assert np.array_equal(ids.cpu().numpy(), got["token"])
    assert not _same_rows(got, want, np.nonzero(~failed)[0])
    # the default budget serves the same batch in full, and the poll is clean
    ctx.set_limits(max_rounds=64)
    got = run()
    ctx.poll_status()
    assert not _same_rows(got, want, range(256))


def test_philox_mode_matches_u_mode(ctx):
    """u == NULL draws Philox4x32-10 (seed per row, counter = (row, 0,
    rng_offset)); the same call fed those uniforms explicitly gives the same
    rows, and both equal the oracle given them."""
    import torch

    from qwenium_b200 import qsamp

    cfg = W.config2(41, B=48)
    p = cfg["params"].copy()
    rng = np.random.default_rng(41)
    p["seed"] = rng.integers(0, 2**63, size=48, dtype=np.uint64)
    offset = 123456789012
    u = np.array([O.philox_uniform(int(p["seed"][b]), offset, b) for b in range(48)])
    x = torch.from_numpy(cfg["logits"]).cuda()
    hist = torch.from_numpy(cfg["hist"]).cuda()
    a = ctx.sample_batch(x, p, hist=hist, hist_len=cfg["hist_len"], u=None, rng_offset=offset)
    b = ctx.sample_batch(x, p, hist=hist, hist_len=cfg["hist_len"], u=u)
    torch.cuda.synchronize()
    ctx.poll_status()
    ga = a.cpu().numpy().view(qsamp.ROW_RESULT).reshape(-1)
    gb = b.cpu().numpy().view(qsamp.ROW_RESULT).reshape(-1)
    assert not _same_rows(ga, gb, range(48))
    want, _, _, _ = O.oracle_sample(cfg["logits"], p, cfg["hist"], cfg["hist_len"], None, u)
    assert not _same_rows(ga, want, range(48))
    assert ga["drew"].sum() > 0
