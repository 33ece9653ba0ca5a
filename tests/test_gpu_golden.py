"""The CUDA path against the golden fixtures made from the reference
(tests/golden), and the grammar-constrained C3 batch against the oracle.

Tokens must equal the reference's (or share its transformed logit, where
std::sort's order of equal logits is unspecified); draw flags must match.
"""
import numpy as np
import pytest

from golden_cases import TOKEN_CASES, config3, config3_fixture, tie_ok, tokens

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from qwenium_b200 import qsamp

    return qsamp.Context(0)


def gpu_rows(ctx, cfg):
    from test_gpu_parity import run_gpu

    r, _, _ = run_gpu(ctx, cfg)
    return r


@pytest.mark.parametrize("name", sorted(TOKEN_CASES))
def test_gpu_matches_golden_tokens(ctx, oracle_mod, name):
    z = tokens()
    cfg = TOKEN_CASES[name]()
    r = gpu_rows(ctx, cfg)
    _, _, _, lo = oracle_mod.oracle_sample(cfg["logits"], cfg["params"], cfg.get("hist"), cfg.get("hist_len"), None,
                                           cfg["u"], want_logits=True)
    for b in range(len(r)):
        assert tie_ok(lo[b], int(r[b]["token"]), int(z[name + "_token"][b])), (name, b)
        assert int(r[b]["drew"]) == int(z[name + "_drew"][b]), (name, b)


def test_gpu_matches_golden_config3(ctx, oracle_mod):
    z = config3_fixture()
    cfg = config3(extensions=False)
    r = gpu_rows(ctx, cfg)
    _, _, _, lo = oracle_mod.oracle_sample(cfg["logits"], cfg["params"], cfg["hist"], cfg["hist_len"], cfg["masks"],
                                           cfg["u"], want_logits=True)
    for b in range(len(r)):
        assert tie_ok(lo[b], int(r[b]["token"]), int(z["token"][b])), b


def test_gpu_config3_with_extensions(ctx, oracle_mod):
    """C3 as specified (frequency / presence penalties on): every field
    against the oracle, with the top-16 survivor list."""
    from test_gpu_parity import check

    check(ctx, oracle_mod, config3(extensions=True))
