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


@pytest.mark.parametrize("fmt", [22, 21, 16, 18, 23])  # IQ2_S, IQ3_S, IQ2_XXS, IQ3_XXS, IQ4_XS
def test_iq_banks_need_whole_16_row_groups(fmt):
    # the IQ formats are stored in 16-row groups; other row counts are refused before any device
    # call (so this runs without a GPU)
    import ctypes

    import numpy as np

    from coachwhip_b200 import _lib

    blk = {22: 82, 21: 110, 16: 66, 18: 98, 23: 136}[fmt]
    n, k = 40, 256
    data = np.zeros(n * blk, dtype=np.uint8)
    d = _lib.MatrixDesc(fmt, n, k, 1, n * blk, data.ctypes.data)
    h = ctypes.c_void_p()
    assert _lib.lib().cwx_bank_create(0, ctypes.byref(d), ctypes.byref(h)) == _lib.EUNSUPPORTED
    assert b"multiple of 16 rows" in _lib.lib().cwx_last_error()
