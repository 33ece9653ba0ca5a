"""Sampling straight from the output head's device tensor.

The server's batched decode reads each slot's logits row back to the host
(ForwardPassBase::get_output_logits_for_slot, forward_pass_base.cpp:138-158)
and samples it there (http_server.cpp:298-306). Here the logits come from an
output-head GEMM on the device -- hidden states [B][D] times the head weight
[V][D], the [B][V] row-major result a column-major ggml tensor with
ne[0] = V is in memory -- and qsamp_sample reads that tensor where it lies:
no device-to-host copy of the logits. The result must equal, bit for bit,
the C restatement run on a host copy of the same logits. Also covered: a
head whose rows are padded past V (a vocabulary rounded up for the GEMM,
row_stride > V) and a bf16 head output.
"""
import numpy as np
import pytest

from qwenium_b200 import workloads as W

pytestmark = pytest.mark.gpu

FIELDS = ("token", "position", "n_keep", "drew", "sum_exp", "sum_keep", "max_logit", "prob")


@pytest.fixture(scope="module")
def ctx():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from qwenium_b200 import qsamp

    return qsamp.Context(0)


def head_logits(B, D, V, V_pad, seed, dtype):
    """The output head on the device: hidden [B][D] @ weight[V_pad][D]^T,
    bf16 operands, fp32 (or bf16) logits [B][V_pad]; the first V columns
    are the vocabulary."""
    import torch

    g = torch.Generator(device="cuda").manual_seed(seed)
    hidden = torch.randn((B, D), generator=g, device="cuda", dtype=torch.float32).to(torch.bfloat16)
    weight = (torch.randn((V_pad, D), generator=g, device="cuda", dtype=torch.float32) * (3.0 / D**0.5)).to(
        torch.bfloat16)
    out = torch.matmul(hidden, weight.t())  # bf16 GEMM
    return out.to(dtype) if dtype == torch.float32 else out


def params_for(B, seed):
    rng = np.random.default_rng(seed)
    p = W.default_params(B)
    p["temperature"] = rng.uniform(0.3, 1.2, B).astype(np.float32)
    p["top_k"] = rng.choice([0, 20, 40, 100], B)
    p["top_p"] = rng.uniform(0.8, 1.0, B).astype(np.float32)
    p["repetition_penalty"] = 1.1
    return p


@pytest.mark.parametrize("V,V_pad,bf16", [(151936, 151936, False), (151655, 151936, False), (262144, 262144, True)])
def test_sample_from_head_output(ctx, oracle_mod, V, V_pad, bf16):
    import torch

    from qwenium_b200 import qsamp

    B, D, H = 16, 1024, 64
    out = head_logits(B, D, V, V_pad, seed=V + V_pad, dtype=torch.bfloat16 if bf16 else torch.float32)
    logits = out[:, :V]  # a view: row stride V_pad, no copy
    assert logits.stride(0) == V_pad
    params = params_for(B, V)
    rng = np.random.default_rng(V)
    hist = rng.integers(0, V, (B, H)).astype(np.int32)
    hl = np.full(B, H, np.int32)
    seeds = np.arange(B, dtype=np.uint32) + 3
    u = W.uniforms_for(seeds)
    dev = logits.view(torch.int16) if bf16 else logits
    res = ctx.sample_batch(dev, params, hist=torch.from_numpy(hist).cuda(), hist_len=hl, u=u)
    torch.cuda.synchronize()
    ctx.poll_status()
    got = res.cpu().numpy().view(qsamp.ROW_RESULT).reshape(-1)
    # the check: the same logits on the host, through the C restatement
    host = logits.contiguous().cpu()
    x = host.view(torch.int16).numpy().view(np.uint16) if bf16 else host.numpy()
    want, _, _, _ = oracle_mod.oracle_sample(np.ascontiguousarray(x), params, hist, hl, None, u, bf16=bf16)
    bad = []
    for b in range(B):
        for f in FIELDS:
            g, w = got[b][f], want[b][f]
            ok = (int(g) == int(w)) if f in FIELDS[:4] else (
                np.float32(g).view(np.uint32) == np.float32(w).view(np.uint32) or (np.isnan(g) and np.isnan(w)))
            if not ok:
                bad.append((b, f, g, w))
    assert not bad, f"{len(bad)} mismatches, first {bad[:6]}"
