"""The C ABI: both libraries load and export every entry point their headers declare (no GPU)."""

import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared(header):
    src = open(header).read()
    return sorted(set(re.findall(r"^(?:int|const char\*|void|float|uint64_t|int64_t)\s+(\w+)\s*\(", src, re.M)))


def test_libcwx_exports_every_declared_symbol():
    from coachwhip_b200 import _lib

    names = _declared(os.path.join(ROOT, "include", "cwx.h"))
    assert len(names) >= 17
    L = _lib.lib()
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    assert sorted(names) == sorted(_lib.EXPORTS)
    assert L.cwx_version() == 1


def test_liboracle_exports_every_declared_symbol():
    import oracle

    names = _declared(os.path.join(ROOT, "oracle", "cw_oracle.h"))
    L = oracle.lib()
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_library_fails_loudly_without_gpu():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from coachwhip_b200 import CwxError, _lib

    with pytest.raises(CwxError):
        _lib.ctx(0)


def test_product_does_not_import_the_oracle():
    pkg = os.path.join(ROOT, "coachwhip_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h")):
                src = open(os.path.join(dirpath, f)).read()
                assert "import oracle" not in src and "from oracle" not in src and "cw_oracle" not in src, f
