"""qsamp_verify_greedy (batched greedy verification of prompt-lookup drafts)
against the restatement pinned to the reference (tests/test_verify.py)."""
import numpy as np
import pytest

from verify_cases import make_cases, verify_one
from qwenium_b200 import workloads as W

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from qwenium_b200 import qsamp

    return qsamp.Context(0)


@pytest.mark.parametrize("seed,V,bf16", [(11, 1, False), (12, 33, False), (13, 4097, True), (14, W.V_QWEN, False),
                                         (15, W.V_QWEN, True)])
def test_verify_greedy(ctx, seed, V, bf16):
    import torch

    B = 48
    x, drafts, off, eos = make_cases(seed, B, V, bf16=bf16)
    if bf16:
        dx = torch.from_numpy(np.ascontiguousarray(W.f32_to_bf16_bits(x)).view(np.int16)).cuda()
    else:
        dx = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    acc, bonus, has = ctx.verify_greedy(dx, torch.from_numpy(off).cuda(), torch.from_numpy(drafts).cuda(), eos)
    torch.cuda.synchronize()
    got = list(zip(acc.cpu().numpy(), bonus.cpu().numpy(), has.cpu().numpy()))
    for b in range(B):
        want = verify_one(x[off[b]:off[b + 1]], drafts[off[b]:off[b + 1]], eos)
        assert tuple(int(v) for v in got[b]) == want, (b, got[b], want)
