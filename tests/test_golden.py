"""The oracle against the golden fixtures (tests/golden, made from the
reference by tests/golden/make_golden.py). No reference code is needed here:
the fixtures hold the reference's tokens, draw flags and uniforms."""
import numpy as np
import pytest

from golden_cases import TOKEN_CASES, config3, config3_fixture, tie_ok, tokens
from qwenium_b200 import qsamp
from qwenium_b200 import workloads as W


@pytest.mark.parametrize("name", sorted(TOKEN_CASES))
def test_oracle_matches_golden_tokens(oracle_mod, name):
    z = tokens()
    cfg = TOKEN_CASES[name]()
    assert np.array_equal(cfg["u"], z[name + "_u"]), "engine uniforms"
    out, _, _, lo = oracle_mod.oracle_sample(cfg["logits"], cfg["params"], cfg.get("hist"), cfg.get("hist_len"),
                                             None, cfg["u"], want_logits=True)
    for b in range(len(out)):
        assert tie_ok(lo[b], int(out[b]["token"]), int(z[name + "_token"][b])), (name, b)
        assert int(out[b]["drew"]) == int(z[name + "_drew"][b]), (name, b)


def test_config3_fixture_is_consistent():
    z = config3_fixture()
    V = W.V_QWEN
    masks, force = z["masks"], z["force"]
    assert masks.shape == (10, (V + 31) // 32)
    for b in range(10):
        bits = int(np.unpackbits(masks[b].view(np.uint8)).sum())
        if z["n_valid"][b] == 0:  # stuck grammar: EOS string forced, mask cleared
            assert force[b] == W.EOT_ID and bits == 0
        else:
            assert force[b] == -1
            extra = 2 if z["accepting"][b] else 0  # EOS string + eos_token_id (sampling.cpp:66-75)
            assert bits == z["n_valid"][b] + extra
            if z["accepting"][b]:
                for e in (W.EOT_ID, W.IM_END_ID):
                    assert masks[b][e // 32] >> np.uint32(e % 32) & 1


def test_config3_masks_from_host_helper():
    """qsamp_grammar_mask packs the reference's valid ids + EOS rules into the
    same bits the reference left finite."""
    z = config3_fixture()
    b = int(np.nonzero(z["accepting"])[0][0])
    ids = np.nonzero(np.unpackbits(z["masks"][b].view(np.uint8), bitorder="little"))[0]
    ids = ids[(ids != W.EOT_ID) & (ids != W.IM_END_ID)].astype(np.int32)
    m, f = qsamp.grammar_mask(ids, True, W.EOT_ID, W.IM_END_ID, W.V_QWEN)
    assert f == -1 and np.array_equal(m, z["masks"][b])
    m, f = qsamp.grammar_mask(np.zeros(0, np.int32), False, W.EOT_ID, W.IM_END_ID, W.V_QWEN)
    assert f == W.EOT_ID and not m.any()


def test_oracle_matches_golden_config3(oracle_mod):
    z = config3_fixture()
    cfg = config3(extensions=False)
    out, _, _, lo = oracle_mod.oracle_sample(cfg["logits"], cfg["params"], cfg["hist"], cfg["hist_len"],
                                             cfg["masks"], cfg["u"], want_logits=True)
    for b in range(len(out)):
        assert tie_ok(lo[b], int(out[b]["token"]), int(z["token"][b])), b
