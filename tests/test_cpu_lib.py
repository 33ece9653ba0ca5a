"""CPU-side checks of the product library: it loads, exports every entry
point include/qsamp.h declares, and its host helpers follow the reference's
grammar/pruning rules (sampling.cpp:12-81). No GPU needed."""
import os
import re
import struct
import tempfile

import numpy as np
import pytest

from qwenium_b200 import build as qbuild
from qwenium_b200 import qsamp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def lib():
    qbuild.build()
    return qsamp.load()


def declared():
    src = open(os.path.join(ROOT, "include", "qsamp.h")).read()
    return sorted(set(re.findall(r"\b(qsamp_[a-z_0-9]+)\s*\(", src)))


def test_exports_every_declared_symbol(lib):
    names = declared()
    assert set(names) == set(qsamp.EXPORTS), names
    for n in names:
        assert hasattr(lib, n), n


def test_row_structs_match_oracle():
    import sys

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    assert O.ROW_PARAMS == qsamp.ROW_PARAMS
    assert O.RESULT.itemsize == qsamp.ROW_RESULT.itemsize


def test_pack_ids_and_and(lib):
    m = qsamp.pack_ids([0, 5, 31, 32, 99, -1, 100, 5], 100)
    assert m.shape == (4,)
    assert m[0] == (1 | 1 << 5 | 1 << 31) and m[1] == 1 and m[3] == 1 << 3
    a = qsamp.mask_and(m, qsamp.pack_ids([5, 99], 100))
    assert a.tolist() == [1 << 5, 0, 0, 1 << 3]


def test_grammar_mask_rules(lib):
    # valid ids, not accepting: exactly the ids
    m, f = qsamp.grammar_mask([1, 2], False, 7, 9, 40)
    assert f == -1 and m[0] == 0b110
    # accepting: the first EOS string and eos_token_id join (sampling.cpp:66-75)
    m, f = qsamp.grammar_mask([1], True, 7, 9, 40)
    assert f == -1 and m[0] == (1 << 1 | 1 << 7 | 1 << 9)
    # stuck grammar: forced EOS string (sampling.cpp:40-60)
    m, f = qsamp.grammar_mask([], True, 7, 9, 40)
    assert f == 7 and not m.any()
    # stuck, no EOS string in the vocab: nothing forced, all masked
    m, f = qsamp.grammar_mask([], False, -1, 9, 40)
    assert f == -1 and not m.any()


def test_find_eos_string(lib):
    vocab = ["a", "<|im_end|>", "<|endoftext|>", "b"]
    assert qsamp.find_eos_string(vocab) == 1
    assert qsamp.find_eos_string(["x", "<|endoftext|>"]) == 1
    assert qsamp.find_eos_string(["x", "y"]) == -1


def test_keep_list_file(lib):
    d = tempfile.mkdtemp()
    p = os.path.join(d, "keep.bin")
    with open(p, "wb") as f:
        f.write(struct.pack("<I", 3) + struct.pack("<3I", 2, 40, 7))
    m = qsamp.keep_list_mask(p, 64)
    assert m[0] == (1 << 2 | 1 << 7) and m[1] == 1 << 8
    with open(p, "wb") as f:
        f.write(struct.pack("<I", 3) + struct.pack("<1I", 2))
    with pytest.raises(qsamp.QsampError):
        qsamp.keep_list_mask(p, 64)
    with pytest.raises(qsamp.QsampError):
        qsamp.keep_list_mask(os.path.join(d, "missing.bin"), 64)


def test_adapter_compiles_against_reference_headers(tmp_path):
    """qwenium_b200/adapter/cuda_sampler.cpp is a qwenium::Sampler subclass:
    it must compile against the reference's own src/sampling headers."""
    import subprocess

    import oracle as O

    if not O.reference_root():
        pytest.skip("reference headers not present")
    inc = os.path.join(O.reference_root(), "src", "sampling")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run(["g++", "-std=c++17", "-O2", "-Wall", "-Wextra", "-I", inc, "-I", os.path.join(root, "include"),
                        "-c", os.path.join(root, "qwenium_b200", "adapter", "cuda_sampler.cpp"),
                        "-o", str(tmp_path / "cuda_sampler.o")], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    assert "warning" not in r.stderr, r.stderr
