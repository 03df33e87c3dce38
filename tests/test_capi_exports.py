"""The C-ABI library loads (no GPU needed) and exports every entry point
declared in include/axb.h; the ctypes table covers exactly those."""

import os
import re
import subprocess

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "axb.h")
LIB = os.path.join(ROOT, "axiomlm_b200", "libaxb.so")


def _declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(axb_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(LIB):
        from axiomlm_b200 import build

        build.build(verbose=False)
    from axiomlm_b200 import _lib

    return _lib.load()


def test_header_declares_entry_points():
    names = _declared()
    assert "axb_qgemm" in names and "axb_runner_step" in names and len(names) >= 25


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", LIB], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (axb_[a-z0-9_]+)$", out, flags=re.M))
    missing = [n for n in _declared() if n not in exported]
    assert not missing, missing
    for n in _declared():
        assert hasattr(lib, n)


def test_ctypes_table_matches_header(lib):
    from axiomlm_b200 import _lib

    assert sorted(_lib.exported_symbols()) == _declared()


def test_host_calls_without_gpu(lib):
    # pure host arithmetic entry points work without a device
    assert lib.axb_version() >= 100
    assert lib.axb_q4t_words_bytes(4096, 4096) == 4096 * 4096 // 2
    assert lib.axb_q4t_scales_bytes(4096, 4096, 128, 1) == 4096 * 32 * 2
    assert lib.axb_q4t_scales_bytes(40, 256, 64, 2) == 3 * 4 * 16 * 2 * 2


def test_invalid_arguments_raise(lib):
    from axiomlm_b200 import _lib

    with pytest.raises(_lib.AxbError):
        _lib.call("axb_q4t_pack", None, 16, 100, 64, 1, 0, None, None, None)
