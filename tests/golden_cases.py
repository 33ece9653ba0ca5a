"""The cases of tests/golden/*.npz: each regenerates its inputs from seeds
(qwenium_b200.workloads) exactly as tests/golden/make_golden.py did, so the
fixtures only hold what the reference returned."""
import os

import numpy as np

from qwenium_b200 import workloads as W

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _no_ext(cfg):
    cfg["params"]["frequency_penalty"] = 0.0
    cfg["params"]["presence_penalty"] = 0.0
    return cfg


TOKEN_CASES = {
    "config1_s1": lambda: W.config1(1),
    "config1_s3": lambda: W.config1(3),
    "config1_greedy": lambda: W.config1(1, greedy=True),
    "config2_b10": lambda: _no_ext(W.config2(2, B=10)),
    "config2_s7_b16": lambda: _no_ext(W.config2(7, B=16)),
    "config5_b16": lambda: W.config5(5, B=16),
}


def tokens():
    return np.load(os.path.join(GOLDEN, "golden_tokens.npz"))


def config3_fixture():
    return np.load(os.path.join(GOLDEN, "config3.npz"))


def config3(extensions):
    z = config3_fixture()
    return W.config3(z["masks"], z["force"], extensions=extensions)


def tie_ok(lo_row, a, b):
    """Two ids whose transformed logits are equal: std::sort leaves their
    order unspecified (the reference may return either)."""
    return a == b or lo_row[a] == lo_row[b]
