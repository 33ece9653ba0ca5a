"""Exhaustive CPU pins of the deterministic scalar math (qs_math.h).

qs_expf must equal glibc's expf (what the reference's sampler calls) on every
float the kernels feed it (x = l - max in [-104, 0]); qs_tanhf must equal the
correctly rounded tanh, (float)tanhl, on every float. The kernels compile the
same header with separately rounded double intrinsics, so these host results
are the device results.
"""
import os
import subprocess
import tempfile

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
NPARTS = max(1, min(16, os.cpu_count() or 1))


@pytest.fixture(scope="module")
def checker():
    d = tempfile.mkdtemp(prefix="qs_math_")
    exe = os.path.join(d, "math_check")
    subprocess.run(["gcc", "-O2", "-ffp-contract=off", "-o", exe, os.path.join(HERE, "math_check.c"), "-lm"],
                   check=True)
    return exe


def _run_parts(exe, what):
    procs = [subprocess.Popen([exe, what, str(i), str(NPARTS)], stdout=subprocess.PIPE, text=True)
             for i in range(NPARTS)]
    bad = 0
    for p in procs:
        out, _ = p.communicate()
        assert p.returncode == 0, out
        last = [ln for ln in out.splitlines() if ln.startswith("bad=")][-1]
        bad += int(last.split("=")[1])
        if last != "bad=0":
            print(out)
    return bad


def test_expf_matches_glibc_on_whole_domain(checker):
    assert _run_parts(checker, "expf") == 0


def test_tanhf_correctly_rounded_on_all_floats(checker):
    assert _run_parts(checker, "tanh") == 0


def test_run_add_matches_sequential_float_loop(checker):
    """qs_run_add (a run of equal terms added in O(1) per binade, used by the
    cluster kernel's walks over bins whose logits are all equal) against the
    plain loop `S = S + t; if (S >= stop) break;` on random runs, including
    exact round-half-to-even ties and binade crossings."""
    procs = [subprocess.Popen([checker, "runadd", str(seed), "20000"], stdout=subprocess.PIPE, text=True)
             for seed in range(NPARTS)]
    for p in procs:
        out, _ = p.communicate()
        assert p.returncode == 0 and out.strip().endswith("bad=0"), out


def test_run_add_d_matches_sequential_double_loop(checker):
    """qs_run_add_d (the double form, used for the cumulative weights of the
    discrete draw over runs of equal probabilities) against `S = S + t; if (S
    >= stop) break;` in double, including ties and binade crossings."""
    procs = [subprocess.Popen([checker, "runaddd", str(seed), "20000"], stdout=subprocess.PIPE, text=True)
             for seed in range(NPARTS)]
    for p in procs:
        out, _ = p.communicate()
        assert p.returncode == 0 and out.strip().endswith("bad=0"), out


def test_expf_tab_matches_qs_expf(checker):
    """qs_expf_tab (the kernels' form: shared-memory table, no special-case
    branches) equals qs_expf on every float in [-104, 0] and at -inf."""
    assert _run_parts(checker, "expftab") == 0


def test_integer_scalings_match_float_definitions(checker):
    """qs_fixed40(t) = (uint64)(t * 2^40) and qs_kround(p, g) = rintf(p *
    2^(23-g)) with its half-way and >= 2^24 flags, on every float in [0, 1]
    (qs_kround at eight binades)."""
    assert _run_parts(checker, "scale") == 0
