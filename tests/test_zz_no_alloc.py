"""The allocation-free entry point, qsamp_sample_static, against qsamp_sample.

Some callers cannot allocate device memory when they sample (a serving engine
that reserves all device memory up front, a plugin host that forbids
cudaMalloc), so they cannot create a qsamp context. qsamp_sample_static serves
them from a fixed static device array. Its results must equal those of the
context-based entry point exactly, on two calls in a row (the second call
finds the first call's contents in the shared array). This file sorts last so
that a run stopping at the first failure has already run every other test.
"""
import numpy as np
import pytest

from qwenium_b200 import workloads as W

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _inputs(torch, cfg):
    x = cfg["logits"]
    dx = torch.from_numpy(x.view(np.int16) if cfg["bf16"] else x).cuda()
    hist = torch.from_numpy(cfg["hist"]).cuda() if cfg["hist"] is not None else None
    return dx, hist


def _two_caps():
    """bf16 rows with two soft-cap values: the static scratch holds one
    soft-cap table, so the rows with the second cap compute tanh per logit."""
    cfg = W.config4(42, B=6)
    cfg["params"]["softcap"] = np.where(np.arange(6) % 2 == 0, 30.0, 20.0).astype(np.float32)
    return cfg


CASES = {
    "config2": lambda: W.config2(31, B=12),
    "config4": lambda: W.config4(41, B=6),
    "config1": lambda: W.config1(51),
    "bf16-two-softcaps": _two_caps,
    # more rows than the launch has clusters: rows come from the row queue
    "rows-exceed-clusters": lambda: W.config2(33, B=96),
}


@pytest.mark.parametrize("ids_only", [False, True], ids=["ids+results", "ids-only"])
@pytest.mark.parametrize("name", list(CASES))
def test_static_entry_matches_context_entry(torch_cuda, name, ids_only):
    """ids_only: no out_results, so the row results go to the static scratch."""
    torch = torch_cuda
    from qwenium_b200 import qsamp

    cfg = CASES[name]()
    dx, hist = _inputs(torch, cfg)
    B = dx.shape[0]
    ctx = qsamp.Context(0)
    ref_ids = torch.empty(B, dtype=torch.int32, device="cuda")
    ref_res = ctx.sample_batch(dx, cfg["params"], hist=hist, hist_len=cfg["hist_len"], u=cfg["u"], out_ids=ref_ids)
    torch.cuda.synchronize()
    want_ids = ref_ids.cpu().numpy()
    want_res = ref_res.cpu().numpy()
    for call in range(2):
        ids = torch.full((B,), -7, dtype=torch.int32, device="cuda")
        res = None if ids_only else torch.zeros((B, qsamp.ROW_RESULT.itemsize), dtype=torch.uint8, device="cuda")
        qsamp.sample_static(dx, cfg["params"], hist=hist, hist_len=cfg["hist_len"], u=cfg["u"], out_ids=ids,
                            out_results=res)
        torch.cuda.synchronize()
        assert np.array_equal(ids.cpu().numpy(), want_ids), f"call {call}: ids differ"
        if res is not None:
            assert np.array_equal(res.cpu().numpy(), want_res), f"call {call}: row results differ"
    ctx.close()


def test_static_entry_rejects_too_many_rows(torch_cuda):
    torch = torch_cuda
    from qwenium_b200 import qsamp

    B = qsamp.STATIC_MAX_ROWS + 1
    dx = torch.zeros((B, 8), dtype=torch.float32, device="cuda")
    ids = torch.empty(B, dtype=torch.int32, device="cuda")
    with pytest.raises(qsamp.QsampError, match="at most 4096 rows"):
        qsamp.sample_static(dx, W.default_params(B), out_ids=ids)
