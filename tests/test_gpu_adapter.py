"""The drop-in C++ adapter (qwenium_b200/adapter: CudaTemperatureSampler and
CudaGreedySampler, subclasses of the reference's qwenium::Sampler) against
the reference's own TemperatureSampler / GreedySampler, side by side.

oracle/_ref/adapter_check is built by oracle/Makefile where the reference
tree exists and travels prebuilt; it compares ids, the logits each sampler
leaves behind (bit for bit) and the state of both engines after every call,
over full-vocabulary top-p, top-k + top-p with a growing history, greedy, a
pruning keep-set, a JSON-grammar walk and empty logits."""
import os
import subprocess

import pytest

from qwenium_b200 import workloads as W

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CHECK = os.path.join(ROOT, "oracle", "_ref", "adapter_check")


def test_adapter_matches_reference_samplers(tmp_path):
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    if not os.path.exists(CHECK):
        pytest.skip("oracle/_ref/adapter_check not built (needs the reference tree)")
    gbnf = tmp_path / "json.gbnf"
    gbnf.write_text(W.JSON_GBNF)
    r = subprocess.run([CHECK, str(gbnf)], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "ALL AGREE" in r.stdout
