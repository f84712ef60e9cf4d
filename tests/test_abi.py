"""CPU: the C-ABI library loads and exports every symbol include/malaga_b200.h declares."""
import os
import re
import subprocess

import pytest

from conftest import gpu_available

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "malaga_b200.h")


def declared() -> list[str]:
    text = open(HEADER).read()
    return sorted(set(re.findall(r"MGB_API\s+[^;(]*?\b(mgb_\w+)\s*\(", text)))


def test_header_declares_the_boundary():
    names = declared()
    for n in ("mgb_open", "mgb_close", "mgb_encode", "mgb_greedy", "mgb_greedy_logits", "mgb_last_error",
              "mgb_argmax_noalloc"):
        assert n in names


def test_library_exports_every_declared_symbol():
    from malaga_b200 import _lib

    lib = _lib.load(build_if_missing=True)
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True, check=True)
    exported = set(re.findall(r"\bT (mgb_\w+)", out.stdout))
    for n in declared():
        assert n in exported, n
        assert getattr(lib, n) is not None
    # the Python bindings cover the header
    assert set(_lib.SIGNATURES) == set(declared())


@pytest.mark.skipif(gpu_available(), reason="checks the no-device error path")
def test_open_without_a_gpu_fails_with_a_message(model):
    from malaga_b200 import Engine, MgbError

    with pytest.raises(MgbError) as e:
        Engine(model("tiny", "q8_0"))
    assert "device" in str(e.value).lower()


def test_library_is_built_for_sm_100a_only():
    from malaga_b200 import build

    flags = " ".join(build.NVCC_FLAGS)
    assert "arch=compute_100a,code=sm_100a" in flags and "-fmad=false" in flags
